"""Isotropic gate frontend (``_iso_kdn_gate_precumsum_paired``,
lit_gpt/kdn_ops/iso_kdn_chunk.py:1396): the CUDA operator against the
reference's own kernels (``tests/golden/iso_gate.npz``) and against the fp64
oracle at other shapes, dtypes and strides; the reference's validation on CPU.

Tolerances: fp32 outputs and gradients 1e-5 normalised max-abs error (the
kernels evaluate softplus with the hardware base-2 exponential and logarithm,
as the reference does); outputs stored in bf16 by contract (dg_raw for a bf16
g_raw, domega_r_raw for a bf16 omega_r_raw) 8e-3 (one bf16 rounding).
"""
import os

import numpy as np
import pytest
import torch

import oracle
from kdn_b200.iso_kdn_chunk import _iso_kdn_gate_precumsum_paired

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
NAMES = ("g_raw", "omega_r_raw", "omega_bias", "r_bias", "A_log", "dt_bias", "initial_precision_param")


def nmax(x, ref):
    x, ref = x.detach().double().cpu(), ref.detach().double().cpu()
    return ((x - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()


def run(inputs, cot, wmin, rmin, gbf, wbf, needs=(True,) * 7, wr_pad=0):
    """Forward + backward through the operator; returns (outputs, grads)."""
    dev = "cuda"
    leaves = []
    for i, t in enumerate(inputs):
        t = t.to(dev)
        if i == 0:
            t = t.to(torch.bfloat16 if gbf else torch.float32)
        elif i == 1:
            t = t.to(torch.bfloat16 if wbf else torch.float32)
            if wr_pad:  # a strided view: rows of 2H + wr_pad, the first 2H used
                B, T, H2 = t.shape
                big = torch.zeros(B, T, H2 + wr_pad, dtype=t.dtype, device=dev)
                big[..., :H2] = t
                t = big[..., :H2]
        else:
            t = t.float()
        leaves.append(t.detach().requires_grad_(needs[i]))
    outs = _iso_kdn_gate_precumsum_paired(*leaves, wmin, rmin)
    pairs = [(o, c.to(dev)) for o, c in zip(outs, cot) if c is not None]
    torch.autograd.backward([o for o, _ in pairs], [c for _, c in pairs])
    torch.cuda.synchronize()
    return [o.detach() for o in outs], [l.grad for l in leaves]


def check(outs, grads, ref_outs, ref_grads, gbf, wbf, needs=(True,) * 7):
    for o, r in zip(outs, ref_outs):
        assert nmax(o, r) < 1e-5
    for i, (g, r) in enumerate(zip(grads, ref_grads)):
        if not needs[i]:
            assert g is None
            continue
        bf = (i == 0 and gbf) or (i == 1 and wbf)
        assert nmax(g, r) < (8e-3 if bf else 1e-5), NAMES[i]


@pytest.mark.gpu
@pytest.mark.parametrize("ci", [0, 1])
def test_gate_matches_reference_kernels(ci):
    with np.load(os.path.join(GOLDEN, "iso_gate.npz")) as z:
        d = {k: torch.from_numpy(z[k]) for k in z.files}
    p = f"c{ci}_"
    B, T, H, K, gbf, wbf, wmin, rmin = d[p + "meta"].tolist()
    inputs = [d[p + n] for n in ("g_raw", "omega_r_raw", "omega_bias", "r_bias", "A_log", "dt_bias", "param")]
    cot = [d[p + n] for n in ("dg_pre", "da", "domega", "dr", "dinit")]
    outs, grads = run(inputs, cot, float(wmin), float(rmin), bool(gbf), bool(wbf))
    ref_outs = [d[p + n] for n in ("g_cumsum", "a", "omega", "r", "initial_precision")]
    ref_grads = [d[p + n] for n in ("dg_raw", "domega_r_raw", "domega_bias", "dr_bias", "dA_log", "ddt_bias", "dparam")]
    check(outs, grads, ref_outs, ref_grads, bool(gbf), bool(wbf))


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H,K,gbf,wbf,wr_pad", [
    (2, 300, 3, 128, True, True, 0),   # ragged last chunk, bf16 inputs
    (1, 64, 5, 64, False, False, 6),   # K = 64, strided omega_r_raw
    (3, 129, 2, 128, False, True, 2),
    (4, 4096, 18, 128, True, False, 0),  # config 1 shape
])
def test_gate_matches_oracle(B, T, H, K, gbf, wbf, wr_pad):
    inputs, cot = oracle.make_iso_gate_inputs(B, T, H, K, seed=B * 1000 + T,
                                              g_dtype=torch.bfloat16 if gbf else torch.float32,
                                              wr_dtype=torch.bfloat16 if wbf else torch.float32)
    outs, grads = run(inputs, cot, 1e-3, 0.01, gbf, wbf, wr_pad=wr_pad)
    ref_outs, ref_grads = oracle.iso_gate_grads(inputs, cot, 1e-3, 0.01)
    check(outs, grads, ref_outs, ref_grads, gbf, wbf)


@pytest.mark.gpu
def test_gate_partial_cotangents_and_grads():
    """Only the gate prefix and the gain outputs feed the loss, and only some
    inputs need gradients: the others come back None, missing cotangents act
    as zeros (set_materialize_grads(False) in the reference)."""
    B, T, H, K = 2, 100, 3, 128
    inputs, cot = oracle.make_iso_gate_inputs(B, T, H, K, seed=7)
    cot = (cot[0], cot[1], None, None, None)
    needs = (True, False, False, True, True, True, False)
    outs, grads = run(inputs, cot, 0.0, 0.01, False, False, needs=needs)
    ref_outs, ref_grads = oracle.iso_gate_grads(inputs, cot, 0.0, 0.01)
    check(outs, grads, ref_outs, ref_grads, False, False, needs=needs)


@pytest.mark.gpu
def test_gate_empty_sequence():
    inputs, cot = oracle.make_iso_gate_inputs(2, 0, 3, 64, seed=3)
    outs, grads = run(inputs, (None, None, None, None, cot[4]), 0.0, 0.01, False, False)
    ref_outs, ref_grads = oracle.iso_gate_grads(inputs, (None, None, None, None, cot[4]), 0.0, 0.01)
    assert outs[0].shape == (2, 0, 3, 64) and outs[1].shape == (2, 0, 3)
    assert nmax(outs[4], ref_outs[4]) < 1e-5
    assert nmax(grads[6], ref_grads[6]) < 1e-5
    for g in grads[2:6]:
        assert torch.count_nonzero(g) == 0


def test_gate_validation_messages():
    """The reference's checks run before any device work (CPU tensors here)."""
    B, T, H, K = 1, 8, 2, 64
    args = [torch.zeros(B, T, H, K), torch.zeros(B, T, 2 * H), torch.zeros(H), torch.zeros(H), torch.zeros(H),
            torch.zeros(H * K), torch.zeros(H)]
    with pytest.raises(ValueError, match="g_raw must have shape"):
        _iso_kdn_gate_precumsum_paired(torch.zeros(B, T, H), *args[1:], 0.0, 0.01)
    with pytest.raises(ValueError, match="omega_r_raw must have shape"):
        _iso_kdn_gate_precumsum_paired(args[0], torch.zeros(B, T, H), *args[2:], 0.0, 0.01)
    with pytest.raises(ValueError, match="dt_bias must have shape"):
        _iso_kdn_gate_precumsum_paired(*args[:5], torch.zeros(H), args[6], 0.0, 0.01)
    with pytest.raises(ValueError, match="CUDA-only"):
        _iso_kdn_gate_precumsum_paired(*args, 0.0, 0.01)


@pytest.mark.gpu
def test_gate_gain_scan_composition():
    """The isotropic mixer's wiring (lit_gpt/iso_kdn.py:277-304): gate frontend
    -> iso_kdn_gain -> _chunk_kda_precumsum_paired, backward through all
    three, against one fp64 autograd graph of the oracle.  This checks the
    paired gate-cotangent exchange between the scan and the frontend.
    Tolerance: the bf16 scan's normalised max-abs bar (1.2e-2; bf16 gradients
    after forgiving their own rounding) for every per-token tensor, 2e-2 for
    the parameter gradients (sums over every token)."""
    from kdn_b200.iso_kdn_chunk import _chunk_kda_precumsum_paired, iso_kdn_gain

    B, T, H, K = 1, 150, 2, 128
    d = oracle.make_iso_inputs(B, T, H, seed=41)
    gate_in, _ = oracle.make_iso_gate_inputs(B, T, H, K, seed=42, g_dtype=torch.bfloat16, wr_dtype=torch.bfloat16)
    # about -1 nat of gate per 64-token chunk
    gate_in = ((gate_in[0].float() * 0.5 - 3.0).bfloat16(),) + tuple(gate_in[1:])
    dO = d["dO"].bfloat16().float()
    wmin, rmin = 0.0, 0.01
    G = [t.to("cuda").detach().requires_grad_(True) for t in gate_in]
    S = {n: d[n].to("cuda").detach().requires_grad_(True) for n in ("q", "k", "v")}
    g_cumsum, a, omega, r, ip = _iso_kdn_gate_precumsum_paired(*G, wmin, rmin)
    beta = iso_kdn_gain(a, omega, r, ip, head_dim=K, out_dtype=torch.float32, info_scale=float(K))
    o = _chunk_kda_precumsum_paired(S["q"], S["k"], S["v"], g_cumsum, beta)
    o.backward(dO.to("cuda"))
    Gr = [t.detach().double().requires_grad_(True) for t in gate_in]
    Sr = {n: d[n].detach().double().requires_grad_(True) for n in ("q", "k", "v")}
    g_r, a_r, omega_r, r_r, ip_r = oracle.iso_gate(*Gr, wmin, rmin)
    beta_r = oracle.iso_gain(a_r, omega_r, r_r, ip_r, 1.0)[0]
    o_r, _ = oracle.iso_scan(Sr["q"], Sr["k"], Sr["v"], g_r, beta_r)
    (o_r * dO.double()).sum().backward()

    def err(x, ref):
        bf = x.dtype == torch.bfloat16
        x, ref = x.detach().double().cpu(), ref.detach().double().cpu()
        excess = (x - ref).abs()
        if bf:  # a bf16 output: forgive its own rounding
            excess = (excess - 2.0 ** -8 * ref.abs()).clamp_min(0)
        return (excess.max() / ref.abs().max().clamp_min(1e-30)).item()

    errs = {"o": err(o, o_r)}
    for name, x, y in zip(NAMES, G, Gr):
        errs["d" + name] = err(x.grad, y.grad)
    for n in ("q", "k", "v"):
        errs["d" + n] = err(S[n].grad, Sr[n].grad)
    from test_gpu_parity import BF16_TOL, log_errors

    log_errors("iso_frontend_gain_scan_composition", errs, {})
    # per-token tensors at the bf16 scan's bar; parameter gradients (sums over
    # every token of the batch) at the north star's 2e-2
    params = ('dA_log', 'ddt_bias', 'domega_bias', 'dr_bias', 'dinitial_precision_param')
    bad = {k: v for k, v in errs.items() if not v < (2e-2 if k in params else BF16_TOL)}
    assert not bad, (bad, errs)
