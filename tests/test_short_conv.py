"""Short causal depthwise convolution with SiLU (``kdn_b200.short_conv``: the
packed q/k/v ``qkv_causal_conv1d`` of the isotropic mixer and the diagonal
mixer's ``_fixed_short_conv``).

* CPU: the float64 oracle (``oracle.short_conv`` and its autograd) agrees with
  the reference's own kernels run under Triton's interpreter
  (``tests/golden/short_conv.npz``, made by ``tests/golden/make_conv_golden.py``).
* GPU: the CUDA kernels agree with the fixture and with the oracle on larger
  cases (the mixers' widths, bf16 and fp32, sequence ends inside a run,
  absent cotangents), forward and backward; the validation raises the
  reference's messages.
Tolerance: normalised max-abs error 1e-2 for bf16-typed tensors (their own
rounding), 1e-5 for fp32 ones; the weight gradient (a sum over every token)
1e-4 for fp32 inputs and 1e-2 for bf16 inputs, whose pre-activation the
reference's backward recomputes in bf16 (iso_kdn_chunk.py:343; measured
1.2e-3 against the oracle).
"""
import os

import numpy as np
import pytest
import torch

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "short_conv.npz")


def nmax(x, ref):
    x, ref = x.detach().double().cpu(), ref.detach().double().cpu()
    return ((x - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()


def tol_of(t, summed=False, x_bf16=False):
    if t.dtype == torch.bfloat16 or (summed and x_bf16):
        return 1e-2
    return 1e-4 if summed else 1e-5


def cases():
    if not os.path.exists(GOLDEN):
        return []
    z = np.load(GOLDEN)
    return sorted({k[: -len("_meta")] for k in z.files if k.endswith("_meta")})


def load(name):
    z = np.load(GOLDEN)
    B, T, D, xbf, wbf = (int(v) for v in z[name + "_meta"])

    def get(key, bf):
        t = torch.from_numpy(z[name + "_" + key].copy())
        return t.view(torch.bfloat16) if bf else t

    d = {k: get(k, xbf) for k in ("x", "dq", "dk", "dv", "q", "k", "v", "dx")}
    d.update({k: get(k, wbf) for k in ("w", "dw")})
    return d


def oracle_qkv(x, w, dys):
    xl, wl = x.double().requires_grad_(True), w.double().requires_grad_(True)
    y = oracle.short_conv(xl, wl)
    D = x.shape[-1] // 3
    outs = (y[..., :D], y[..., D:2 * D], y[..., 2 * D:])
    used = [(o, c.double()) for o, c in zip(outs, dys) if c is not None]
    torch.autograd.backward([o for o, _ in used], [c for _, c in used])
    return [o.detach() for o in outs], xl.grad, wl.grad


def test_golden_fixture_present():
    assert cases(), "tests/golden/short_conv.npz is missing (tests/golden/make_conv_golden.py makes it)"


@pytest.mark.parametrize("name", cases())
def test_oracle_matches_reference_kernels(name):
    d = load(name)
    (q, k, v), dx, dw = oracle_qkv(d["x"], d["w"], (d["dq"], d["dk"], d["dv"]))
    for got, ref in ((d["q"], q), (d["k"], k), (d["v"], v), (d["dx"], dx)):
        assert nmax(got, ref) < tol_of(got)
    assert nmax(d["dw"], dw) < tol_of(d["dw"], summed=True, x_bf16=d["x"].dtype == torch.bfloat16)


@pytest.mark.gpu
@pytest.mark.parametrize("name", cases())
def test_kernels_match_reference_kernels(name):
    from kdn_b200.short_conv import qkv_causal_conv1d

    d = load(name)
    x, w = d["x"].cuda().requires_grad_(True), d["w"].cuda().requires_grad_(True)
    outs = qkv_causal_conv1d(x, w)
    torch.autograd.backward(list(outs), [d[n].cuda() for n in ("dq", "dk", "dv")])
    for got, ref in zip(outs, (d["q"], d["k"], d["v"])):
        assert got.dtype == ref.dtype and nmax(got, ref) < tol_of(got)
    assert nmax(x.grad, d["dx"]) < tol_of(x.grad)
    assert nmax(w.grad, d["dw"]) < tol_of(w.grad, summed=True, x_bf16=d["x"].dtype == torch.bfloat16)


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,D,xdt,wdt,present", [(4, 1000, 256, torch.bfloat16, torch.float32, (1, 1, 1)),
                                                   (1, 35, 128, torch.float32, torch.float32, (1, 0, 1)),
                                                   (2, 3, 64, torch.bfloat16, torch.bfloat16, (0, 1, 0))])
def test_qkv_kernels_match_oracle(B, T, D, xdt, wdt, present):
    from kdn_b200.short_conv import qkv_causal_conv1d

    gen = torch.Generator().manual_seed(B + T + D)
    x = torch.randn(B, T, 3 * D, generator=gen).to(xdt)
    w = (torch.randn(3 * D, 4, generator=gen) * 0.5).to(wdt)
    dys = [torch.randn(B, T, D, generator=gen).to(xdt) if p else None for p in present]
    xl, wl = x.cuda().requires_grad_(True), w.cuda().requires_grad_(True)
    outs = qkv_causal_conv1d(xl, wl)
    used = [(o, c.cuda()) for o, c in zip(outs, dys) if c is not None]
    torch.autograd.backward([o for o, _ in used], [c for _, c in used])
    refs, rdx, rdw = oracle_qkv(x, w, dys)
    for got, ref in zip(outs, refs):
        assert nmax(got, ref) < tol_of(got)
    assert nmax(xl.grad, rdx) < tol_of(xl.grad)
    assert nmax(wl.grad, rdw) < tol_of(wl.grad, summed=True)


@pytest.mark.gpu
def test_fixed_short_conv_matches_oracle():
    from kdn_b200.short_conv import fixed_short_conv

    conv = torch.nn.Conv1d(256, 256, 4, groups=256, bias=False, padding=3).cuda()
    x = torch.randn(2, 129, 256, device="cuda").bfloat16().requires_grad_(True)
    y = fixed_short_conv(conv, x)
    dy = torch.randn_like(y)
    y.backward(dy)
    xl = x.detach().double().cpu().requires_grad_(True)
    wl = conv.weight.detach().double().cpu().reshape(256, 4).requires_grad_(True)
    ref = oracle.short_conv(xl, wl)
    ref.backward(dy.double().cpu())
    assert nmax(y, ref) < 1e-2
    assert nmax(x.grad, xl.grad) < 1e-2
    assert nmax(conv.weight.grad.reshape(256, 4), wl.grad) < 1e-4


@pytest.mark.gpu
def test_validation_matches_reference_messages():
    from kdn_b200.short_conv import qkv_causal_conv1d

    x = torch.randn(1, 8, 12, device="cuda")
    with pytest.raises(ValueError, match="rank-3"):
        qkv_causal_conv1d(x[0], torch.randn(12, 4, device="cuda"))
    with pytest.raises(ValueError, match="multiple of 3"):
        qkv_causal_conv1d(x[..., :10], torch.randn(10, 4, device="cuda"))
    with pytest.raises(ValueError, match="packed weight must be"):
        qkv_causal_conv1d(x, torch.randn(12, 3, device="cuda"))
    with pytest.raises(TypeError, match="bfloat16 or float32"):
        qkv_causal_conv1d(x.half(), torch.randn(12, 4, device="cuda"))
