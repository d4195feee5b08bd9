"""Diagonal gate / noise frontend (``_diag_kdn_frontend_precumsum_paired``,
lit_gpt/kdn_ops/diag_kdn_chunk.py:2471): the CUDA operator against the
reference's own kernels (``tests/golden/diag_gate.npz``) and against the fp64
oracle at other shapes and cotangent patterns; the reference's validation on CPU.

Tolerances: fp32 outputs and gradients 1e-5 normalised max-abs error (softplus
and alpha from the hardware base-2 exponential and logarithm, as the
reference's Triton lowering does); the bf16 gradients (dretention_raw,
domega_raw, dr_raw carry their input's dtype) 8e-3, one bf16 rounding.
"""
import os

import numpy as np
import pytest
import torch

import oracle
from kdn_b200.diag_kdn_chunk import _diag_kdn_frontend_precumsum_paired

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
INPUTS = ("retention_raw", "omega_raw", "r_raw", "A_log", "dt_bias", "param")
COTANGENTS = ("d_g_cumsum", "d_alpha", "d_omega", "d_r", "d_init")
OUTPUTS = ("g_cumsum", "alpha", "omega", "r", "initial_precision")
GRADS = ("dretention_raw", "domega_raw", "dr_raw", "dA_log", "ddt_bias", "dparam")
BF16_GRADS = (0, 1, 2)


def nmax(x, ref):
    x, ref = x.detach().double().cpu(), ref.detach().double().cpu()
    return ((x - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()


def run(inputs, cot, needs=(True,) * 6):
    dev = "cuda"
    leaves = [t.to(dev).detach().requires_grad_(n) for t, n in zip(inputs, needs)]
    outs = _diag_kdn_frontend_precumsum_paired(*leaves)
    pairs = [(o, c.to(dev)) for o, c in zip(outs, cot) if c is not None]
    if pairs and any(needs):
        torch.autograd.backward([o for o, _ in pairs], [c for _, c in pairs])
    torch.cuda.synchronize()
    return [o.detach() for o in outs], [l.grad for l in leaves]


def check(outs, grads, ref_outs, ref_grads, expect_none=()):
    for name, o, r in zip(OUTPUTS, outs, ref_outs):
        assert o.dtype == torch.float32
        assert nmax(o, r) < 1e-5, name
    for i, (g, r) in enumerate(zip(grads, ref_grads)):
        if i in expect_none:
            assert g is None, GRADS[i]
            continue
        assert g is not None, GRADS[i]
        assert nmax(g, r) < (8e-3 if i in BF16_GRADS else 1e-5), GRADS[i]


@pytest.mark.gpu
@pytest.mark.parametrize("ci", [0, 1])
def test_diag_frontend_matches_reference_kernels(ci):
    with np.load(os.path.join(GOLDEN, "diag_gate.npz")) as z:
        d = {k: torch.from_numpy(z[k]) for k in z.files}
    p = f"c{ci}_"
    inputs = [d[p + n] for n in INPUTS]
    inputs = [t.to(torch.bfloat16) if i < 3 else t for i, t in enumerate(inputs)]
    cot = [d[p + n] for n in COTANGENTS]
    outs, grads = run(inputs, cot)
    assert grads[0].dtype == grads[1].dtype == grads[2].dtype == torch.bfloat16
    check(outs, grads, [d[p + n] for n in OUTPUTS], [d[p + n] for n in GRADS])


@pytest.mark.gpu
@pytest.mark.parametrize(
    "B,T,H,K",
    [(1, 1, 1, 64), (1, 32, 1, 128), (2, 97, 3, 64), (1, 1000, 4, 128)],
)
def test_diag_frontend_matches_oracle(B, T, H, K):
    inputs, cot = oracle.make_diag_gate_inputs(B, T, H, K, seed=B * 1000 + T + K)
    outs, grads = run(inputs, cot)
    ref_outs, ref_grads = oracle.diag_gate_grads(inputs, cot)
    check(outs, grads, ref_outs, ref_grads)


@pytest.mark.gpu
@pytest.mark.parametrize(
    "present,needs",
    [
        ((True, False, False, False, False), (True, False, False, True, True, False)),
        ((False, True, False, True, False), (True, True, True, False, True, True)),
        ((False, False, True, False, True), (True, True, False, True, False, True)),
        ((True, True, True, True, True), (False, True, True, False, False, True)),
    ],
)
def test_diag_frontend_partial_cotangents(present, needs):
    """Absent cotangents count as zero; a gradient is None when its input does
    not need one or its cotangent (or, for the decay inputs, both decay
    cotangents) is absent (diag_kdn_chunk.py:2280-2443)."""
    inputs, cot = oracle.make_diag_gate_inputs(2, 70, 2, 128, seed=5)
    cot = [c if p else None for c, p in zip(cot, present)]
    outs, grads = run(inputs, cot, needs)
    ref_outs, ref_grads = oracle.diag_gate_grads(inputs, cot)
    has_decay = present[0] or present[1]
    expect_none = [i for i in range(6) if not needs[i]]
    if not has_decay:
        expect_none += [0, 3, 4]
    if not present[2]:
        expect_none.append(1)
    if not present[3]:
        expect_none.append(2)
    if not present[4]:
        expect_none.append(5)
    check(outs, grads, ref_outs, ref_grads, expect_none=set(expect_none))


def test_diag_frontend_validation_messages():
    """The reference's validation order and messages (diag_kdn_chunk.py:2171-2215)
    as far as they are reachable without a GPU."""
    inputs, _ = oracle.make_diag_gate_inputs(1, 4, 2, 64)
    with pytest.raises(TypeError, match="retention_raw must be a torch.Tensor"):
        _diag_kdn_frontend_precumsum_paired(None, *inputs[1:])
    with pytest.raises(ValueError, match="retention_raw must be a CUDA tensor"):
        _diag_kdn_frontend_precumsum_paired(*inputs)


@pytest.mark.gpu
def test_diag_frontend_gain_scan_composition():
    """The diagonal mixer's wiring (lit_gpt/diag_kdn.py:315-342): frontend ->
    _diag_kdn_gain (with the raw noise logits) -> chunk_kalman, backward
    through all three, against one fp64 autograd graph of the oracle.  This
    checks the paired gate-cotangent exchange between chunk_kalman and the
    frontend (natural-log coordinates before the reverse 32-token prefix).
    Tolerance: the bf16 scan's normalised max-abs bar (1.2e-2; bf16 gradients
    after forgiving their own rounding) for every per-token tensor, 2e-2 for
    the parameter gradients (sums over every token)."""
    from kdn_b200.diag_kdn_chunk import _diag_kdn_gain, chunk_kalman

    B, T, H, K = 1, 100, 2, 128
    d = oracle.make_diag_inputs(B, T, H, seed=31)
    gate_in, _ = oracle.make_diag_gate_inputs(B, T, H, K, seed=32)
    # milder decays than the frontend-only cases: chunk products stay above the
    # exact-gate regime of the bf16 scan
    gate_in = ((gate_in[0].float() * 0.5 - 2.0).bfloat16(),) + tuple(gate_in[1:3]) + (gate_in[3] * 0.5,) + tuple(gate_in[4:])
    dO = d["dO"].bfloat16().float()
    scale = K ** -0.5
    # ours
    G = [t.to("cuda").detach().requires_grad_(True) for t in gate_in]
    S = {n: d[n].to("cuda").detach().requires_grad_(True) for n in ("q", "k", "v", "k_gain")}
    g_cumsum, alpha, omega, r, ip = _diag_kdn_frontend_precumsum_paired(*G)
    kappa = _diag_kdn_gain(S["k_gain"], alpha, omega, r, ip, G[1], G[2])
    o = chunk_kalman(S["q"], S["k"], kappa, S["v"], g_cumsum, scale)
    o.backward(dO.to("cuda"))
    # oracle
    Gr = [t.detach().double().requires_grad_(True) for t in gate_in]
    Sr = {n: d[n].detach().double().requires_grad_(True) for n in ("q", "k", "v", "k_gain")}
    g_r, alpha_r, omega_r, r_r, ip_r = oracle.diag_gate(*Gr)
    kappa_r, _ = oracle.diag_gain(Sr["k_gain"], alpha_r, omega_r, r_r, ip_r)
    alpha_mem = oracle.alpha_from_g_cumsum(g_r * oracle.LN2, 32)
    S0 = torch.zeros(B, H, K, K, dtype=torch.float64)
    o_r, _ = oracle.memory_recurrence(Sr["q"], Sr["k"], Sr["v"], alpha_mem, kappa_r, S0, scale)
    (o_r * dO.double()).sum().backward()

    def err(x, ref):
        bf = x.dtype == torch.bfloat16
        x, ref = x.detach().double().cpu(), ref.detach().double().cpu()
        excess = (x - ref).abs()
        if bf:  # a bf16 output: forgive its own rounding
            excess = (excess - 2.0 ** -8 * ref.abs()).clamp_min(0)
        return (excess.max() / ref.abs().max().clamp_min(1e-30)).item()

    errs = {"o": err(o, o_r)}
    for name, a, b in zip(("retention_raw", "omega_raw", "r_raw", "A_log", "dt_bias", "param"), G, Gr):
        errs["d" + name] = err(a.grad, b.grad)
    for n in ("q", "k", "v", "k_gain"):
        errs["d" + n] = err(S[n].grad, Sr[n].grad)
    from test_gpu_parity import BF16_TOL, log_errors

    log_errors("diag_frontend_gain_scan_composition", errs, {})
    # per-token tensors at the bf16 scan's bar; parameter gradients (sums over
    # every token of the batch) at the north star's 2e-2
    params = ('dA_log', 'ddt_bias', 'dparam')
    bad = {k: v for k, v in errs.items() if not v < (2e-2 if k in params else BF16_TOL)}
    assert not bad, (bad, errs)
