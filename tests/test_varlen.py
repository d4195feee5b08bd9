"""Packed variable-length batches (config 4's varlen variant).

The memory scans and the gains run natively over the packed batch (a chunk
table from ``kdn_varlen_plan``): every sequence owns its 64-token chunks and
its gain stream, so each sequence gets the arithmetic of a separate
fixed-length call of that sequence alone, which the parity tests pin to the oracle.  The
comparison bar is therefore tight: normalised max-abs error 1e-5 for fp32
outputs, and one bf16 unit in the last place per element for bf16 outputs
(the chunk-parallel backward sums some partial products with shared-memory
atomics, whose order varies from run to run, so even two identical calls
can round an element differently; the per-head prior's gradient sums the
sequences in another order than a sum of separate calls).  The packed
call is also checked against the float64 oracle directly at the bf16 bars.
"""
import ctypes

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


def agree(x, ref, tol=TOL):
    """fp32: normalised max-abs error below tol; bf16: every element within
    one bf16 ulp of the other call's (plus tol of the largest magnitude)."""
    if x.dtype != torch.bfloat16:
        return nmax(x, ref) < tol
    x, ref = x.detach().double().cpu(), ref.detach().double().cpu()
    return bool(((x - ref).abs() <= ref.abs() * 2.0 ** -7 + tol * ref.abs().max()).all())


def pack(ds, names):
    return {n: torch.cat([d[n] for d in ds], dim=1) for n in names}


def offsets_of(lens):
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    return cu


def test_offsets_validation():
    assert varlen.offsets([0, 3, 10]) == [0, 3, 10]
    assert varlen.offsets(torch.tensor([0, 5])) == [0, 5]
    for bad in ([1, 4], [0], [0, 4, 4], [0, 5, 3]):
        with pytest.raises(ValueError):
            varlen.offsets(bad)


def test_plan_table():
    """kdn_varlen_plan (host code of the library, no GPU): chunk offsets, the
    longest-first order and each chunk's sequence."""
    lens = [70, 5, 128, 64, 1]
    p = varlen.plan(offsets_of(lens), "cpu")
    n, nc = len(lens), sum(-(-x // 64) for x in lens)
    assert (p.num_seqs, p.num_chunks) == (n, nc)
    t = p.table.tolist()
    assert len(t) == 3 * n + 2 + nc
    tok, chunk, order, seq = t[:n + 1], t[n + 1:2 * n + 2], t[2 * n + 2:3 * n + 2], t[3 * n + 2:]
    assert tok == offsets_of(lens)
    assert chunk == offsets_of([-(-x // 64) for x in lens])
    assert order == [2, 0, 3, 1, 4]  # by decreasing length, ties in packed order
    assert seq == [i for i, x in enumerate(lens) for _ in range(-(-x // 64))]
    assert varlen.plan(offsets_of(lens), "cpu") is p  # cached


def test_plan_validation():
    from kdn_b200 import _native as N

    lib = N.load_library()
    nc = ctypes.c_int64(0)
    for bad in ([1, 4], [0, 4, 4], [0, 5, 3]):
        arr = (ctypes.c_int64 * len(bad))(*bad)
        assert lib.kdn_varlen_plan(ctypes.cast(arr, ctypes.c_void_p), len(bad) - 1, None, 0, ctypes.byref(nc)) != 0
    arr = (ctypes.c_int64 * 3)(0, 65, 70)
    assert lib.kdn_varlen_plan(ctypes.cast(arr, ctypes.c_void_p), 2, None, 0, ctypes.byref(nc)) == 0
    assert nc.value == 3
    small = torch.empty(4, dtype=torch.int32)  # 3 * 2 + 2 + 3 = 11 entries needed
    assert lib.kdn_varlen_plan(ctypes.cast(arr, ctypes.c_void_p), 2, small.data_ptr(), 4, ctypes.byref(nc)) != 0


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


# sequences ending inside a chunk, on a chunk boundary, inside the first
# 32-token gate block, single tokens, and many short sequences in a row
LENGTHS = {"mixed": [40, 96, 33, 7], "edges": [64, 1, 65, 63, 128, 32, 31], "many": [3, 17, 9, 70, 2, 5, 64, 11]}


@pytest.mark.gpu
@pytest.mark.parametrize("case", sorted(LENGTHS))
def test_diag_varlen_matches_per_sequence(case):
    lens = LENGTHS[case]
    ds = [oracle.make_diag_inputs(1, n, 2, seed=100 + i) for i, n in enumerate(lens)]
    x = pack(ds, DIAG)
    x["initial_precision"] = ds[0]["initial_precision"]
    cu = offsets_of(lens)
    o, grads = diag_step(x, torch.tensor(cu))
    total = None
    for i, d in enumerate(ds):
        d = dict(d, initial_precision=x["initial_precision"])
        o_i, g_i = diag_step(d)
        sl = slice(cu[i], cu[i + 1])
        assert agree(o[:, sl], o_i), f"seq {i}: o"
        for n in DIAG_GRADS:
            if n != "initial_precision":
                assert agree(grads[n][:, sl], g_i[n]), f"seq {i}: d{n}"
        total = g_i["initial_precision"] if total is None else total + g_i["initial_precision"]
    # the per-head prior collects every sequence's cotangent
    assert nmax(grads["initial_precision"], total) < TOL


ISO = ("q", "k", "v", "g_cumsum", "a", "omega", "r", "dO")
ISO_GRADS = ("q", "k", "v", "g_cumsum", "a", "omega", "r")


def iso_step(x, prec, cu=None):
    L = {n: x[n].to(DEV).clone().requires_grad_(True) for n in ISO_GRADS}
    p = prec.to(DEV).clone().requires_grad_(True)
    if cu is None:
        beta = iso_kdn_gain(L["a"], L["omega"], L["r"], p, head_dim=128, out_dtype=torch.float32)
        o = _chunk_kda_precumsum_paired(L["q"], L["k"], L["v"], L["g_cumsum"], beta)
    else:
        beta = varlen.iso_kdn_gain_varlen(L["a"], L["omega"], L["r"], p, head_dim=128, cu_seqlens=cu,
                                          out_dtype=torch.float32)
        o = varlen.chunk_kda_precumsum_varlen(L["q"], L["k"], L["v"], L["g_cumsum"], beta, cu_seqlens=cu)
    o.float().backward(x["dO"].to(DEV).float())
    torch.cuda.synchronize()
    return o.detach(), dict({n: L[n].grad for n in ISO_GRADS}, prec=p.grad)


@pytest.mark.gpu
@pytest.mark.parametrize("case", sorted(LENGTHS))
def test_iso_varlen_matches_per_sequence(case):
    lens = LENGTHS[case]
    ds = [oracle.make_iso_inputs(1, n, 2, seed=200 + i, dtype=torch.bfloat16) for i, n in enumerate(lens)]
    x = pack(ds, ISO)
    prec = torch.ones(2)
    cu = offsets_of(lens)
    o, grads = iso_step(x, prec, cu)
    total = 0.0
    for i, d in enumerate(ds):
        o_i, g_i = iso_step(d, prec)
        sl = slice(cu[i], cu[i + 1])
        assert agree(o[:, sl], o_i), f"seq {i}: o"
        for n in ISO_GRADS:
            assert agree(grads[n][:, sl], g_i[n]), f"seq {i}: d{n}"
        total = total + g_i["prec"]
    # the per-head prior collects every sequence's cotangent
    assert nmax(grads["prec"], total) < TOL


@pytest.mark.gpu
def test_varlen_validation():
    lens = [40, 30]
    d = oracle.make_diag_inputs(1, 70, 2, seed=7)
    q, k, v = (d[n].to(DEV) for n in ("q", "k", "v"))
    kappa, g = torch.rand(1, 70, 2, 128, device=DEV), d["g_cumsum"].to(DEV)
    with pytest.raises(ValueError, match="cu_seqlens"):
        varlen.chunk_kalman_varlen(q, k, kappa, v, g, 128 ** -0.5, [0, 40, 69])
    with pytest.raises(ValueError):
        varlen.chunk_kalman_varlen(q, k, kappa, v, g, 128 ** -0.5, [0, 40, 40, 70])
    q2 = torch.cat([q, q])
    with pytest.raises(ValueError, match="packed"):
        varlen.chunk_kalman_varlen(q2, torch.cat([k, k]), torch.cat([kappa, kappa]), torch.cat([v, v]),
                                   torch.cat([g, g]), 128 ** -0.5, offsets_of(lens))


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
    cu = offsets_of(lens)
    o, grads = diag_step(x, torch.tensor(cu))
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
