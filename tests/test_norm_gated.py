"""Gated RMS normalisation of the scan output (``kdn_b200.norm_gated``, the
drop-in for flash-linear-attention's ``FusedRMSNormGated`` that both
reference mixers apply before the output projection).

* CPU: the float64 oracle (``oracle.rms_norm_gated`` and its autograd) agrees
  with flash-linear-attention's own kernels run under Triton's interpreter
  (``tests/golden/norm_gated.npz``, made by
  ``tests/golden/make_norm_gated_golden.py``) to the outputs' own rounding.
* GPU: the CUDA kernels through the module agree with the fixture and with
  the oracle on larger cases (the mixers' shapes, both activations, bf16 and
  fp32), forward and backward.
Tolerance: normalised max-abs error 1e-2 for bf16-typed outputs (one bf16
rounding of values up to a few units), 1e-5 for fp32 outputs; the weight
gradient, a sum over every row, 1e-4.
"""
import os

import numpy as np
import pytest
import torch

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "norm_gated.npz")


def nmax(x, ref):
    x, ref = x.detach().double().cpu(), ref.detach().double().cpu()
    return ((x - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()


def tol_of(t):
    return 1e-2 if t.dtype == torch.bfloat16 else 1e-5


def cases():
    if not os.path.exists(GOLDEN):
        return []
    z = np.load(GOLDEN)
    return sorted({k[: -len("_meta")] for k in z.files if k.endswith("_meta")})


def load(name):
    z = np.load(GOLDEN)
    D, xbf, gbf, swish, has_w = (int(v) for v in z[name + "_meta"])

    def get(key, bf):
        if name + "_" + key not in z.files:
            return None
        t = torch.from_numpy(z[name + "_" + key].copy())
        return t.view(torch.bfloat16) if bf else t

    d = {k: get(k, xbf) for k in ("x", "dy", "y", "dx")}
    d.update({k: get(k, gbf) for k in ("g", "dg")})
    d.update({k: get(k, False) for k in ("w", "dw")})
    d["activation"] = "swish" if swish else "sigmoid"
    return d


def oracle_grads(d):
    x, g = d["x"].double().requires_grad_(True), d["g"].double().requires_grad_(True)
    w = None if d["w"] is None else d["w"].double().requires_grad_(True)
    y = oracle.rms_norm_gated(x, g, w, 1e-5, d["activation"])
    y.backward(d["dy"].double())
    return y.detach(), x.grad, g.grad, None if w is None else w.grad


def test_golden_fixture_present():
    assert cases(), "tests/golden/norm_gated.npz is missing (tests/golden/make_norm_gated_golden.py makes it)"


@pytest.mark.parametrize("name", cases())
def test_oracle_matches_reference_kernels(name):
    d = load(name)
    y, dx, dg, dw = oracle_grads(d)
    assert nmax(d["y"], y) < tol_of(d["y"])
    assert nmax(d["dx"], dx) < tol_of(d["dx"])
    assert nmax(d["dg"], dg) < tol_of(d["dg"])
    if dw is not None:
        assert nmax(d["dw"], dw) < 1e-4


def run_ours(x, g, w, dy, activation):
    from kdn_b200.norm_gated import FusedRMSNormGated

    mod = FusedRMSNormGated(x.shape[-1], elementwise_affine=w is not None, eps=1e-5, activation=activation).cuda()
    if w is not None:
        with torch.no_grad():
            mod.weight.copy_(w)
    xl, gl = x.cuda().requires_grad_(True), g.cuda().requires_grad_(True)
    y = mod(xl, gl)
    y.backward(dy.cuda())
    return y, xl.grad, gl.grad, None if w is None else mod.weight.grad


@pytest.mark.gpu
@pytest.mark.parametrize("name", cases())
def test_kernels_match_reference_kernels(name):
    d = load(name)
    y, dx, dg, dw = run_ours(d["x"], d["g"], d["w"], d["dy"], d["activation"])
    assert y.dtype == d["y"].dtype and dx.dtype == d["dx"].dtype and dg.dtype == d["dg"].dtype
    ry, rdx, rdg, rdw = oracle_grads(d)
    for got, ref in ((y, ry), (dx, rdx), (dg, rdg)):
        assert nmax(got, ref) < tol_of(got)
    if dw is not None:
        assert nmax(dw, rdw) < 1e-4 and nmax(dw, d["dw"]) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("shape,D,xdt,gdt,act", [((4, 512, 18), 128, torch.bfloat16, torch.bfloat16, "sigmoid"),
                                                 ((2, 300, 3), 64, torch.bfloat16, torch.float32, "swish"),
                                                 ((1, 7), 128, torch.float32, torch.float32, "sigmoid")])
def test_kernels_match_oracle(shape, D, xdt, gdt, act):
    gen = torch.Generator().manual_seed(D + len(shape))
    x = (torch.randn(*shape, D, generator=gen) * 3).to(xdt)
    g = torch.randn(*shape, D, generator=gen).to(gdt)
    w = 1.0 + 0.2 * torch.randn(D, generator=gen)
    dy = torch.randn(*shape, D, generator=gen).to(xdt)
    y, dx, dg, dw = run_ours(x, g, w, dy, act)
    ry, rdx, rdg, rdw = oracle_grads({"x": x, "g": g, "w": w, "dy": dy, "activation": act})
    for got, ref in ((y, ry), (dx, rdx), (dg, rdg)):
        assert nmax(got, ref) < tol_of(got)
    assert nmax(dw, rdw) < 1e-4
