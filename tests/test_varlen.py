"""Packed variable-length batches (config 4's varlen variant).

The varlen operators must give, sequence by sequence, what the fixed-length
operators give for that sequence alone (which the parity tests pin to the
oracle): the memory state, covariance and chunk-local gate prefix all restart
at each ``cu_seqlens`` boundary.  The packed call runs each sequence as a row
of a padded batch, which rounds a sequence's last partial chunk like a full
chunk, so the comparison uses the bf16 parity tolerance (normalised max-abs
error and relative Frobenius error <= 2e-2); the fp32 gain outputs agree to
1e-5.
"""
import pytest
import torch

import oracle
from kdn_b200 import varlen
from kdn_b200.diag_kdn_chunk import _diag_kdn_gain, chunk_kalman
from kdn_b200.iso_kdn_chunk import _chunk_kda_precumsum_paired, iso_kdn_gain

DEV = "cuda"
TOL = 2e-2


def nmax(x, ref):
    x, ref = x.detach().double().cpu(), ref.detach().double().cpu()
    return ((x - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()


def frob(x, ref):
    x, ref = x.detach().double().cpu(), ref.detach().double().cpu()
    return ((x - ref).norm() / ref.norm().clamp_min(1e-30)).item()


def close(x, ref, tol=TOL):
    return nmax(x, ref) < tol and frob(x, ref) < tol


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


def diag_step(x, cu=None, bucket=1024):
    L = {n: x[n].to(DEV).clone().requires_grad_(n in DIAG_GRADS) for n in DIAG_GRADS + ("omega", "r")}
    scale = 128 ** -0.5
    if cu is None:
        kappa = _diag_kdn_gain(L["k_gain"], L["alpha"], L["omega"], L["r"], L["initial_precision"], L["omega_raw"],
                               L["r_raw"])
        o = chunk_kalman(L["q"], L["k"], kappa, L["v"], L["g_cumsum"], scale)
    else:
        kappa = varlen.diag_kdn_gain_varlen(L["k_gain"], L["alpha"], L["omega"], L["r"], L["initial_precision"],
                                            L["omega_raw"], L["r_raw"], cu, bucket=bucket)
        o = varlen.chunk_kalman_varlen(L["q"], L["k"], kappa, L["v"], L["g_cumsum"], scale, cu, bucket=bucket)
    o.backward(x["dO"].to(DEV))
    torch.cuda.synchronize()
    return o.detach(), {n: L[n].grad for n in DIAG_GRADS}


@pytest.mark.gpu
@pytest.mark.parametrize("bucket", [64, 1024])  # 64: two length groups; 1024: one
def test_diag_varlen_matches_per_sequence(bucket):
    lens = [40, 96, 33, 7]
    ds = [oracle.make_diag_inputs(1, n, 2, seed=100 + i) for i, n in enumerate(lens)]
    x = pack(ds, DIAG)
    x["initial_precision"] = ds[0]["initial_precision"]
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    o, grads = diag_step(x, torch.tensor(cu), bucket)
    for i, d in enumerate(ds):
        d = dict(d, initial_precision=x["initial_precision"])
        o_i, g_i = diag_step(d)
        sl = slice(cu[i], cu[i + 1])
        assert close(o[:, sl], o_i), f"seq {i}: o"
        for n in DIAG_GRADS:
            if n == "initial_precision":
                continue
            assert close(grads[n][:, sl], g_i[n]), f"seq {i}: d{n}"
    # the per-head prior collects every sequence's cotangent (through the
    # bf16 scan's dkappa, hence the bf16 tolerance)
    total = sum(diag_step(dict(d, initial_precision=x["initial_precision"]))[1]["initial_precision"] for d in ds)
    assert close(grads["initial_precision"], total)


ISO = ("q", "k", "v", "g_cumsum", "a", "omega", "r", "dO")
ISO_GRADS = ("q", "k", "v", "g_cumsum", "a", "omega", "r")


def iso_step(x, prec, cu=None, bucket=1024):
    L = {n: x[n].to(DEV).clone().requires_grad_(True) for n in ISO_GRADS}
    p = prec.to(DEV)
    if cu is None:
        beta = iso_kdn_gain(L["a"], L["omega"], L["r"], p, head_dim=128, out_dtype=torch.float32)
        o = _chunk_kda_precumsum_paired(L["q"], L["k"], L["v"], L["g_cumsum"], beta)
    else:
        beta = varlen.iso_kdn_gain_varlen(L["a"], L["omega"], L["r"], p, head_dim=128, cu_seqlens=cu,
                                          out_dtype=torch.float32, bucket=bucket)
        o = varlen.chunk_kda_precumsum_varlen(L["q"], L["k"], L["v"], L["g_cumsum"], beta, cu_seqlens=cu,
                                              bucket=bucket)
    o.float().backward(x["dO"].to(DEV).float())
    torch.cuda.synchronize()
    return o.detach(), {n: L[n].grad for n in ISO_GRADS}


@pytest.mark.gpu
@pytest.mark.parametrize("bucket", [64, 1024])
def test_iso_varlen_matches_per_sequence(bucket):
    lens = [70, 130, 64, 5]
    ds = [oracle.make_iso_inputs(1, n, 2, seed=200 + i, dtype=torch.bfloat16) for i, n in enumerate(lens)]
    x = pack(ds, ISO)
    prec = torch.ones(2)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    o, grads = iso_step(x, prec, cu, bucket)
    for i, d in enumerate(ds):
        o_i, g_i = iso_step(d, prec)
        sl = slice(cu[i], cu[i + 1])
        assert close(o[:, sl], o_i), f"seq {i}: o"
        for n in ISO_GRADS:
            assert close(grads[n][:, sl], g_i[n]), f"seq {i}: d{n}"


@pytest.mark.gpu
def test_diag_varlen_against_the_oracle():
    """The packed call against the float64 oracle directly, sequence by
    sequence (gain + memory recurrence restarting at every boundary): the
    bf16 scan's bars, the few-token bar for a 7-token sequence."""
    from test_gpu_parity import BF16_FTOL, BF16_TOL, check_errors

    lens = [200, 64, 7, 130]
    ds = [oracle.make_diag_inputs(1, n, 2, seed=300 + i) for i, n in enumerate(lens)]
    for d in ds:
        d["dO"] = d["dO"].bfloat16().float()  # chunk_kalman rounds its cotangent to bf16
    x = pack(ds, DIAG)
    x["initial_precision"] = ds[0]["initial_precision"]
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    o, grads = diag_step(x, torch.tensor(cu), 64)
    for i, d in enumerate(ds):
        sl = slice(cu[i], cu[i + 1])
        L = {n: d[n].double().clone().requires_grad_(True) for n in ("q", "k", "v", "k_gain", "alpha", "omega_raw",
                                                                      "r_raw")}
        G = (d["g_cumsum"].double() * oracle.LN2).requires_grad_(True)
        omega = torch.nn.functional.softplus(L["omega_raw"])
        r = 0.01 + torch.nn.functional.softplus(L["r_raw"])
        kappa, _ = oracle.diag_gain(L["k_gain"], L["alpha"], omega, r, x["initial_precision"].double())
        S0 = torch.zeros(1, 2, 128, 128, dtype=torch.float64)
        o_r, _ = oracle.memory_recurrence(L["q"], L["k"], L["v"], oracle.alpha_from_g_cumsum(G, 32), kappa, S0,
                                          128 ** -0.5)
        (o_r * d["dO"].double()).sum().backward()
        got = {"o": o[:, sl], "dg": grads["g_cumsum"][:, sl]}
        ref = {"o": o_r.detach(), "dg": G.grad}
        for n in ("q", "k", "v", "k_gain", "alpha", "omega_raw", "r_raw"):
            got["d" + n], ref["d" + n] = grads[n][:, sl], L[n].grad
        short = lens[i] < 16
        check_errors(f"varlen_diag_seq{i}", got, ref, {"dq", "dk", "dv", "domega_raw", "dr_raw"},
                     2e-2 if short else BF16_TOL, 2e-2 if short else BF16_FTOL)
