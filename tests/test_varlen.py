"""Packed variable-length batches (config 4's varlen variant).

The varlen operators must give, sequence by sequence, what the fixed-length
operators give for that sequence alone (which the parity tests pin to the
oracle): the memory state, covariance and chunk-local gate prefix all restart
at each ``cu_seqlens`` boundary.  Tolerance 1e-5 normalised max-abs error: the
same kernels run on the same values; only the order of a few fp32 atomic
additions inside a CTA may differ between runs.
"""
import pytest
import torch

import oracle
from kdn_b200 import varlen
from kdn_b200.diag_kdn_chunk import _diag_kdn_gain, chunk_kalman
from kdn_b200.iso_kdn_chunk import _chunk_kda_precumsum_paired, iso_kdn_gain

DEV = "cuda"
TOL = 1e-5


def nmax(x, ref):
    x, ref = x.detach().double().cpu(), ref.detach().double().cpu()
    return ((x - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()


def pack(ds, names):
    return {n: torch.cat([d[n] for d in ds], dim=1) for n in names}


def test_offsets_validation():
    assert varlen.offsets([0, 3, 10]) == [0, 3, 10]
    assert varlen.offsets(torch.tensor([0, 5])) == [0, 5]
    for bad in ([1, 4], [0], [0, 4, 4], [0, 5, 3]):
        with pytest.raises(ValueError):
            varlen.offsets(bad)


DIAG = ("q", "k", "v", "g_cumsum", "k_gain", "alpha", "omega", "r", "omega_raw", "r_raw", "dO")
DIAG_GRADS = ("q", "k", "v", "g_cumsum", "k_gain", "alpha", "omega_raw", "r_raw", "initial_precision")


def diag_step(x, cu=None):
    L = {n: x[n].to(DEV).clone().requires_grad_(n in DIAG_GRADS) for n in DIAG_GRADS + ("omega", "r")}
    scale = 128 ** -0.5
    if cu is None:
        kappa = _diag_kdn_gain(L["k_gain"], L["alpha"], L["omega"], L["r"], L["initial_precision"], L["omega_raw"],
                               L["r_raw"])
        o = chunk_kalman(L["q"], L["k"], kappa, L["v"], L["g_cumsum"], scale)
    else:
        kappa = varlen.diag_kdn_gain_varlen(L["k_gain"], L["alpha"], L["omega"], L["r"], L["initial_precision"],
                                            L["omega_raw"], L["r_raw"], cu)
        o = varlen.chunk_kalman_varlen(L["q"], L["k"], kappa, L["v"], L["g_cumsum"], scale, cu)
    o.backward(x["dO"].to(DEV))
    torch.cuda.synchronize()
    return o.detach(), {n: L[n].grad for n in DIAG_GRADS}


@pytest.mark.gpu
def test_diag_varlen_matches_per_sequence():
    lens = [40, 96, 33, 7]
    ds = [oracle.make_diag_inputs(1, n, 2, seed=100 + i) for i, n in enumerate(lens)]
    x = pack(ds, DIAG)
    x["initial_precision"] = ds[0]["initial_precision"]
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    o, grads = diag_step(x, torch.tensor(cu))
    for i, d in enumerate(ds):
        d = dict(d, initial_precision=x["initial_precision"])
        o_i, g_i = diag_step(d)
        sl = slice(cu[i], cu[i + 1])
        assert nmax(o[:, sl], o_i) < TOL, f"seq {i}: o"
        for n in DIAG_GRADS:
            if n == "initial_precision":
                continue
            assert nmax(grads[n][:, sl], g_i[n]) < TOL, f"seq {i}: d{n}"
    # the per-head prior collects every sequence's cotangent
    total = sum(diag_step(dict(d, initial_precision=x["initial_precision"]))[1]["initial_precision"] for d in ds)
    assert nmax(grads["initial_precision"], total) < 1e-4


ISO = ("q", "k", "v", "g_cumsum", "a", "omega", "r", "dO")
ISO_GRADS = ("q", "k", "v", "g_cumsum", "a", "omega", "r")


def iso_step(x, prec, cu=None):
    L = {n: x[n].to(DEV).clone().requires_grad_(True) for n in ISO_GRADS}
    p = prec.to(DEV)
    if cu is None:
        beta = iso_kdn_gain(L["a"], L["omega"], L["r"], p, head_dim=128, out_dtype=torch.float32)
        o = _chunk_kda_precumsum_paired(L["q"], L["k"], L["v"], L["g_cumsum"], beta)
    else:
        beta = varlen.iso_kdn_gain_varlen(L["a"], L["omega"], L["r"], p, head_dim=128, cu_seqlens=cu,
                                          out_dtype=torch.float32)
        o = varlen.chunk_kda_precumsum_varlen(L["q"], L["k"], L["v"], L["g_cumsum"], beta, cu_seqlens=cu)
    o.float().backward(x["dO"].to(DEV).float())
    torch.cuda.synchronize()
    return o.detach(), {n: L[n].grad for n in ISO_GRADS}


@pytest.mark.gpu
def test_iso_varlen_matches_per_sequence():
    lens = [70, 130, 64, 5]
    ds = [oracle.make_iso_inputs(1, n, 2, seed=200 + i, dtype=torch.bfloat16) for i, n in enumerate(lens)]
    x = pack(ds, ISO)
    prec = torch.ones(2)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    o, grads = iso_step(x, prec, cu)
    for i, d in enumerate(ds):
        o_i, g_i = iso_step(d, prec)
        sl = slice(cu[i], cu[i + 1])
        assert nmax(o[:, sl], o_i) < TOL, f"seq {i}: o"
        for n in ISO_GRADS:
            assert nmax(grads[n][:, sl], g_i[n]) < TOL, f"seq {i}: d{n}"
