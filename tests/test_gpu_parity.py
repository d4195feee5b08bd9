"""GPU parity: the sm_100a kernels against the CPU oracle on identical seeded inputs.

Tolerances (stated per the north star):
* gains (fp32 arithmetic): normalised max-abs error <= 1e-4;
* scans, fp32 debug precision (``KDN_B200_PRECISION=fp32``): normalised
  max-abs error <= 1e-4 for o and every gradient;
* scans, bf16 tensor-core precision (the product, the tcgen05 kernels):
  normalised max-abs error < 1.2e-2 and relative Frobenius error < 8e-3 for
  o, the final state and every gradient.  These bars sit about 1.5x above
  the largest errors measured on a B200 over every case here and at the
  benchmarked shapes (8.1e-3 and 5.7e-3, both on the gate cotangent dg;
  typical outputs 3-5e-3), well inside the north star's 2e-2.  The one
  exception is a 3-token sequence, where the normalisation runs over three
  rows only (dg 1.8e-2 / 1.4e-2 measured): it keeps the north star's 2e-2.
normalised max-abs error = max|x - ref| / max|ref|.
"""
import os

import pytest
import torch

import oracle
from kdn_b200.diag_kdn_chunk import _diag_kdn_gain, chunk_kalman
from kdn_b200.iso_kdn_chunk import _chunk_kda_precumsum_paired, iso_kdn_gain

pytestmark = pytest.mark.gpu
DEV = "cuda"


def nmax(x, ref):
    x = x.detach().double().cpu()
    ref = ref.detach().double().cpu()
    return ((x - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()


def frob(x, ref):
    x = x.detach().double().cpu()
    ref = ref.detach().double().cpu()
    return ((x - ref).norm() / ref.norm().clamp_min(1e-30)).item()


@pytest.fixture
def precision(request):
    old = os.environ.get("KDN_B200_PRECISION")
    os.environ["KDN_B200_PRECISION"] = request.param
    yield request.param
    if old is None:
        os.environ.pop("KDN_B200_PRECISION", None)
    else:
        os.environ["KDN_B200_PRECISION"] = old


# ----------------------------------------------------------------------------- gains


# T around the 128-token blocks of the gain kernels; H = 40: two head groups of 32 lanes
@pytest.mark.parametrize("T,H", [(1, 3), (37, 3), (128, 3), (129, 5), (300, 3), (1000, 3), (4096, 18), (300, 40)])
@pytest.mark.parametrize("s", [1.0, 0.5])
def test_iso_gain_fwd_bwd(T, H, s):
    torch.manual_seed(T)
    B = 2
    a = torch.rand(B, T, H) * 0.98 + 0.01
    omega = torch.nn.functional.softplus(torch.randn(B, T, H))
    r = 0.01 + torch.nn.functional.softplus(torch.randn(B, T, H))
    prec = 0.1 + torch.nn.functional.softplus(torch.randn(H))
    dbeta = torch.randn(B, T, H)
    beta_ref, da_ref, dw_ref, dr_ref, dp_ref = oracle.iso_gain_grads(a, omega, r, prec, dbeta, s)
    leaves = [x.to(DEV).requires_grad_(True) for x in (a, omega, r, prec)]
    beta = iso_kdn_gain(*leaves, head_dim=128, info_scale=128 * s)
    beta.backward(dbeta.to(DEV))
    assert nmax(beta, beta_ref) < 1e-5
    for got, ref in zip((x.grad for x in leaves), (da_ref, dw_ref, dr_ref, dp_ref)):
        assert nmax(got, ref) < 1e-4


@pytest.mark.parametrize("T,K", [(1, 128), (70, 128), (200, 64), (513, 128)])
def test_diag_gain_fwd_bwd(T, K):
    torch.manual_seed(T + K)
    B, H = 2, 2
    d = oracle.make_diag_inputs(B, T, H, K=K, V=K, seed=T)
    prec = 0.1 + torch.nn.functional.softplus(torch.randn(H))
    dkappa = torch.randn(B, T, H, K)
    kap_ref, dk_ref, da_ref, dwr_ref, drr_ref, dp_ref = oracle.diag_gain_grads(
        d["k_gain"], d["alpha"], d["omega"], d["r"], prec, d["omega_raw"], d["r_raw"], dkappa
    )
    k = d["k_gain"].to(DEV).requires_grad_(True)
    alpha = d["alpha"].to(DEV).requires_grad_(True)
    p = prec.to(DEV).requires_grad_(True)
    wr = d["omega_raw"].to(DEV).requires_grad_(True)
    rr = d["r_raw"].to(DEV).requires_grad_(True)
    kappa = _diag_kdn_gain(k, alpha, d["omega"].to(DEV), d["r"].to(DEV), p, wr, rr)
    kappa.backward(dkappa.to(DEV))
    assert nmax(kappa, kap_ref) < 1e-4
    assert nmax(k.grad, dk_ref) < 1e-4
    assert nmax(alpha.grad, da_ref) < 1e-4
    assert nmax(p.grad, dp_ref) < 1e-4
    # bf16 outputs: one bf16 rounding
    assert nmax(wr.grad, dwr_ref) < 1e-2
    assert nmax(rr.grad, drr_ref) < 1e-2


def _off16(x):
    """The same values at an address one element past a 16-byte boundary."""
    buf = torch.empty(x.numel() + 1, dtype=x.dtype, device=DEV)
    y = buf[1:].view(x.shape)
    y.copy_(x)
    return y


@pytest.mark.parametrize("T,K", [(200, 128), (77, 64)])
def test_diag_gain_unaligned_rows(T, K):
    """Rows that are not 16-byte aligned take the kernels' 4-byte copy path;
    it must give what the 16-byte path gives."""
    torch.manual_seed(T)
    B, H = 2, 3
    d = oracle.make_diag_inputs(B, T, H, K=K, V=K, seed=T)
    prec = (0.1 + torch.nn.functional.softplus(torch.randn(H))).to(DEV)
    dkappa = torch.randn(B, T, H, K).to(DEV)
    base = {n: d[n].to(DEV) for n in ("k_gain", "alpha", "omega", "r", "omega_raw", "r_raw")}
    outs = []
    for shift in (False, True):
        x = {n: (_off16(v) if shift and n != "r" and n != "r_raw" else v.clone()) for n, v in base.items()}
        if shift:
            assert x["k_gain"].data_ptr() % 16 != 0 and x["omega_raw"].data_ptr() % 16 != 0
        k = x["k_gain"].requires_grad_(True)
        alpha = x["alpha"].requires_grad_(True)
        p = prec.clone().requires_grad_(True)
        wr = x["omega_raw"].requires_grad_(True)
        rr = x["r_raw"].requires_grad_(True)
        kappa = _diag_kdn_gain(k, alpha, x["omega"], x["r"], p, wr, rr)
        kappa.backward(_off16(dkappa) if shift else dkappa)
        outs.append([kappa.detach(), k.grad, alpha.grad, p.grad, wr.grad.float(), rr.grad.float()])
    for a, b in zip(*outs):
        assert nmax(b, a) < 1e-6


# ----------------------------------------------------------------------------- scans


def run_iso(d, dO):
    leaves = {n: d[n].to(DEV).requires_grad_(True) for n in ("q", "k", "v", "g_cumsum", "beta")}
    o = _chunk_kda_precumsum_paired(leaves["q"], leaves["k"], leaves["v"], leaves["g_cumsum"], leaves["beta"])
    o.backward(dO.to(DEV))
    return o, {n: leaves[n].grad for n in leaves}


def run_diag(d, dO, kappa, scale):
    q, k, v, g = (d[n].to(DEV).requires_grad_(True) for n in ("q", "k", "v", "g_cumsum"))
    kap = kappa.to(DEV).requires_grad_(True)
    o = chunk_kalman(q, k, kap, v, g, scale)
    o.backward(dO.to(DEV))
    return o, {"q": q.grad, "k": k.grad, "kappa": kap.grad, "v": v.grad, "g_cumsum": g.grad}


def nmax_rounded(x, ref):
    """Like nmax, for an output whose dtype is bf16 by contract: each element
    may differ from the exact value by its own rounding to bf16 (relative
    2^-8, the unit roundoff of an 8-bit significand), so that much is
    forgiven per element before the maximum is taken.  fp32-typed outputs
    get no such allowance (plain ``nmax``)."""
    x = x.detach().double().cpu()
    ref = ref.detach().double().cpu()
    excess = ((x - ref).abs() - 2.0 ** -8 * ref.abs()).clamp_min(0)
    return (excess.max() / ref.abs().max().clamp_min(1e-30)).item()


def fmt(d):
    return "{" + ", ".join(f"{k}: {v:.3g}" for k, v in d.items()) + "}"


def log_errors(case, errs, ferrs):
    """Append the measured errors of one case to ``$KDN_TEST_ERRLOG`` (JSON
    lines) when that variable is set: the tolerances below were set from
    these records."""
    path = os.environ.get("KDN_TEST_ERRLOG")
    if not path:
        return
    import json

    with open(path, "a") as f:
        f.write(json.dumps({"case": case, "nmax": errs, "frob": ferrs}) + "\n")


def check_errors(case, got, ref, bf16_typed, tol, ftol=None):
    """Normalised max-abs error of every entry of ``got`` against ``ref``
    (bf16-typed entries after their own rounding, see ``nmax_rounded``) below
    ``tol``, and relative Frobenius error below ``ftol`` when given."""
    errs = {k: (nmax_rounded(got[k], ref[k]) if k in bf16_typed else nmax(got[k], ref[k])) for k in got}
    ferrs = {k: frob(got[k], ref[k]) for k in got}
    log_errors(case, errs, ferrs)
    bad = {k: v for k, v in errs.items() if not v < tol}
    assert not bad, f"over {tol}: {fmt(bad)}; all: {fmt(errs)}"
    if ftol is not None:
        badf = {k: v for k, v in ferrs.items() if not v < ftol}
        assert not badf, f"frobenius over {ftol}: {fmt(badf)}; all: {fmt(ferrs)}"


def check(o, grads, ref, names, tol, ftol=None, case=None):
    got = {"o": o}
    for n in names:
        got["dg" if n == "g_cumsum" else "d" + n] = grads[n]
    bf16_typed = {k for k, x in got.items() if x.dtype == torch.bfloat16}
    if case is None:  # the running test's id, parameters included
        case = os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0].split("::")[-1]
    check_errors(case, got, {k: ref[k] for k in got}, bf16_typed, tol, ftol)


# fp32: the SIMT debug kernels; bf16: the tcgen05 product kernels
BF16_TOL, BF16_FTOL = 1.2e-2, 8e-3
TOL = {"fp32": (1e-4, None), "bf16": (BF16_TOL, BF16_FTOL)}
SHORT_TOL = {"fp32": (1e-4, None), "bf16": (2e-2, 2e-2)}  # sequences of a few tokens


@pytest.mark.parametrize("precision", ["fp32", "bf16"], indirect=True)
# decay 2.4 (ln alpha about -1.9 per token): chunks whose gate stays within
# the fast path's range around the reference row while the chunk's total
# decay, 2^g_L, underflows fp32 (the last row's state term must stay finite)
@pytest.mark.parametrize("B,T,H,decay", [(1, 130, 2, 1.0), (2, 64, 1, 1.0), (1, 3, 1, 1.0), (1, 200, 1, 8.0),
                                         (1, 192, 2, 2.4)])
def test_iso_scan(precision, B, T, H, decay):
    d = oracle.make_iso_inputs(B, T, H, seed=T + B, decay_scale=decay)
    ref = oracle.scan_grads("iso", {n: d[n] for n in ("q", "k", "v", "g_cumsum", "beta")}, d["dO"])
    o, grads = run_iso(d, d["dO"])
    tol, ftol = (SHORT_TOL if T < 16 else TOL)[precision]
    check(o, grads, ref, ("q", "k", "v", "g_cumsum", "beta"), tol, ftol)


@pytest.mark.parametrize("precision", ["fp32", "bf16"], indirect=True)
# decay 8 puts every chunk on the exact-gate path (gate range ~150 bits around the reference row)
@pytest.mark.parametrize("B,T,H,decay", [(1, 70, 2, 1.0), (2, 32, 1, 1.0), (1, 5, 1, 1.0), (1, 100, 1, 8.0),
                                         (1, 192, 2, 2.4)])
def test_diag_scan(precision, B, T, H, decay):
    d = oracle.make_diag_inputs(B, T, H, seed=T + 7, decay_scale=decay)
    # the kernel rounds the fp32 cotangent to bf16 (diag_kdn_chunk.py:3277); feed one that is exact in bf16
    d["dO"] = d["dO"].bfloat16().float()
    kappa = oracle.diag_gain(d["k_gain"].double(), d["alpha"].double(), d["omega"].double(), d["r"].double(),
                             d["initial_precision"].double())[0].float()
    scale = 128 ** -0.5
    ref = oracle.scan_grads("diag", {"q": d["q"], "k": d["k"], "kappa": kappa, "v": d["v"], "g_cumsum": d["g_cumsum"]},
                            d["dO"], scale=scale)
    o, grads = run_diag(d, d["dO"], kappa, scale)
    tol, ftol = TOL[precision]
    check(o, grads, ref, ("q", "k", "kappa", "v", "g_cumsum"), tol, ftol)


# Narrower heads than the kernels' 128 channels (the reference's diagonal
# scan takes K = V in {64, 128}, its isotropic one K <= 256): the operators
# run them zero-padded to 128 and slice the results.
@pytest.mark.parametrize("precision", ["fp32", "bf16"], indirect=True)
@pytest.mark.parametrize("K,V", [(64, 64), (64, 128), (128, 64), (96, 32)])
def test_iso_scan_narrow_heads(precision, K, V):
    d = oracle.make_iso_inputs(1, 150, 2, K=K, V=V, seed=K + V)
    ref = oracle.scan_grads("iso", {n: d[n] for n in ("q", "k", "v", "g_cumsum", "beta")}, d["dO"])
    o, grads = run_iso(d, d["dO"])
    assert o.shape == (1, 150, 2, V)
    tol, ftol = TOL[precision]
    check(o, grads, ref, ("q", "k", "v", "g_cumsum", "beta"), tol, ftol)


@pytest.mark.parametrize("precision", ["fp32", "bf16"], indirect=True)
def test_diag_scan_k64(precision):
    d = oracle.make_diag_inputs(1, 150, 2, K=64, V=64, seed=64)
    d["dO"] = d["dO"].bfloat16().float()
    kappa = oracle.diag_gain(d["k_gain"].double(), d["alpha"].double(), d["omega"].double(), d["r"].double(),
                             d["initial_precision"].double())[0].float()
    scale = 64 ** -0.5
    ref = oracle.scan_grads("diag", {"q": d["q"], "k": d["k"], "kappa": kappa, "v": d["v"], "g_cumsum": d["g_cumsum"]},
                            d["dO"], scale=scale)
    o, grads = run_diag(d, d["dO"], kappa, scale)
    assert o.shape == (1, 150, 2, 64)
    tol, ftol = TOL[precision]
    check(o, grads, ref, ("q", "k", "kappa", "v", "g_cumsum"), tol, ftol)


# Longer sequences (17 to 66 chunks): the sequential passes' multi-stage
# pipelines wrap around their stage rings several times.
@pytest.mark.parametrize("precision", ["bf16"], indirect=True)
@pytest.mark.parametrize("B,T,H", [(1, 1100, 2), (1, 2100, 1)])
def test_iso_scan_long(precision, B, T, H):
    d = oracle.make_iso_inputs(B, T, H, seed=T + 11)
    ref = oracle.scan_grads("iso", {n: d[n] for n in ("q", "k", "v", "g_cumsum", "beta")}, d["dO"])
    o, grads = run_iso(d, d["dO"])
    tol, ftol = TOL[precision]
    check(o, grads, ref, ("q", "k", "v", "g_cumsum", "beta"), tol, ftol)


@pytest.mark.parametrize("precision", ["bf16"], indirect=True)
@pytest.mark.parametrize("B,T,H", [(1, 600, 2), (1, 1050, 1)])
def test_diag_scan_long(precision, B, T, H):
    d = oracle.make_diag_inputs(B, T, H, seed=T + 13)
    d["dO"] = d["dO"].bfloat16().float()
    kappa = oracle.diag_gain(d["k_gain"].double(), d["alpha"].double(), d["omega"].double(), d["r"].double(),
                             d["initial_precision"].double())[0].float()
    scale = 128 ** -0.5
    ref = oracle.scan_grads("diag", {"q": d["q"], "k": d["k"], "kappa": kappa, "v": d["v"], "g_cumsum": d["g_cumsum"]},
                            d["dO"], scale=scale)
    o, grads = run_diag(d, d["dO"], kappa, scale)
    tol, ftol = TOL[precision]
    check(o, grads, ref, ("q", "k", "kappa", "v", "g_cumsum"), tol, ftol)


# ----------------------------------------------------------------------------- continuation (sequence parallelism)


def _iso_full_reference(d, prec):
    names = ("q", "k", "v", "g_cumsum", "a", "omega", "r")
    L = {n: d[n].double().clone().requires_grad_(True) for n in names}
    P = prec.double().clone().requires_grad_(True)
    beta, _, _ = oracle.iso_gain(L["a"], L["omega"], L["r"], P, 1.0)
    qh, kh = oracle.l2norm(L["q"]), oracle.l2norm(L["k"])
    alpha = oracle.alpha_from_g_cumsum(L["g_cumsum"] * oracle.LN2, 64)
    S0 = torch.zeros(qh.shape[0], qh.shape[2], 128, 128, dtype=torch.float64)
    o, _ = oracle.memory_recurrence(qh, kh, L["v"], alpha, beta[..., None] * kh, S0, 128 ** -0.5)
    (o * d["dO"].double()).sum().backward()
    ref = {"o": o.detach(), "dprec": P.grad}
    ref.update({"d" + n: L[n].grad for n in names})
    # the operator's gate cotangent is taken in natural-log coordinates, G = ln2 * g
    ref["dg"] = ref.pop("dg_cumsum") / oracle.LN2
    return ref


@pytest.mark.parametrize("precision,T,cuts", [("fp32", 256, (128, 192)), ("bf16", 256, (128, 192)),
                                               ("bf16", 2200, (64, 128))], indirect=["precision"])
def test_iso_segments_with_carried_state(precision, T, cuts):
    """Three segments chained through (S, p) reproduce one full-sequence call
    (at T = 2200 the last segment is 33 chunks long)."""
    from kdn_b200.sequence_parallel import iso_segment

    d = oracle.make_iso_inputs(1, T, 2, seed=21)
    prec = torch.tensor([1.0, 0.7])
    ref = _iso_full_reference(d, prec)
    names = ("q", "k", "v", "g_cumsum", "a", "omega", "r")
    L = {n: d[n].to(DEV).requires_grad_(True) for n in names}
    P = prec.to(DEV).requires_grad_(True)
    outs, S, p = [], None, None
    for s0, s1 in zip((0,) + cuts, cuts + (T,)):
        seg = [L[n][:, s0:s1] for n in names]
        o, S, p = iso_segment(*seg, P, S, p, head_dim=128)
        outs.append(o)
    o = torch.cat(outs, 1)
    o.backward(d["dO"].to(DEV))
    grads = {n: L[n].grad for n in names}
    grads["prec"] = P.grad
    tol, ftol = TOL[precision]
    check(o, grads, ref, names + ("prec",), tol, ftol)


@pytest.mark.parametrize("precision", ["fp32", "bf16"], indirect=True)
def test_diag_segments_with_carried_state(precision):
    from kdn_b200.sequence_parallel import diag_segment

    d = oracle.make_diag_inputs(1, 160, 2, seed=22)
    d["dO"] = d["dO"].bfloat16().float()
    prec = torch.tensor([1.0, 0.6])
    names = ("q", "k", "v", "g_cumsum", "k_gain")
    # reference: the full-sequence oracle (gain with alpha from g, then the memory scan)
    Lr = {n: d[n].double().clone().requires_grad_(True) for n in names}
    Pr = prec.double().clone().requires_grad_(True)
    alpha_r = oracle.alpha_from_g_cumsum(Lr["g_cumsum"] * oracle.LN2, 32)
    kappa_r, _ = oracle.diag_gain(Lr["k_gain"], alpha_r, d["omega"].double(), d["r"].double(), Pr)
    S0 = torch.zeros(1, 2, 128, 128, dtype=torch.float64)
    o_r, _ = oracle.memory_recurrence(Lr["q"], Lr["k"], Lr["v"], alpha_r, kappa_r, S0, 128 ** -0.5)
    (o_r * d["dO"].double()).sum().backward()
    ref = {"o": o_r.detach(), "dprec": Pr.grad, **{"d" + n: Lr[n].grad for n in names}}
    # ours: the gain takes alpha from the same g so both paths share it
    L = {n: d[n].to(DEV).requires_grad_(True) for n in names}
    P = prec.to(DEV).requires_grad_(True)
    alpha = oracle.alpha_from_g_cumsum(d["g_cumsum"].double() * oracle.LN2, 32).float().to(DEV)
    omega, r, wr, rr = (d[n].to(DEV) for n in ("omega", "r", "omega_raw", "r_raw"))
    outs, S, p = [], None, None
    for s0, s1 in ((0, 64), (64, 96), (96, 160)):
        o, S, p = diag_segment(L["q"][:, s0:s1], L["k"][:, s0:s1], L["v"][:, s0:s1], L["g_cumsum"][:, s0:s1],
                               L["k_gain"][:, s0:s1].contiguous(), alpha[:, s0:s1].contiguous(),
                               omega[:, s0:s1].contiguous(), r[:, s0:s1].contiguous(), P,
                               wr[:, s0:s1].contiguous(), rr[:, s0:s1].contiguous(), S, p)
        outs.append(o)
    o = torch.cat(outs, 1)
    o.backward(d["dO"].to(DEV))
    grads = {n: L[n].grad for n in names}
    grads["prec"] = P.grad
    tol, ftol = TOL[precision]
    # the memory scan's gate cotangent has no reference here (alpha enters the gain separately)
    check(o, grads, ref, ("q", "k", "v", "k_gain", "prec"), tol, ftol)


def test_sp_nccl_two_gpus(tmp_path):
    """Sequence parallelism over NCCL between two GPUs (skipped on one GPU)."""
    import subprocess
    import sys

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import socket

    with socket.socket() as sock:  # a free port for the rendezvous
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(here, "sp_nccl_worker.py"), str(tmp_path)]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600,
                         env={**os.environ, "NCCL_NVLS_ENABLE": "0"})
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    assert "sp nccl ok" in res.stdout
    assert "sp two-pass nccl ok" in res.stdout
