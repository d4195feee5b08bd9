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
