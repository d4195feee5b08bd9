"""Generate the golden fixtures that pin the CPU oracle to the reference.

The reference ships no tests or known-answer vectors, so its two independent
PyTorch oracles are the ground truth:

* ``lit_gpt/kdn_ops/iso_kdn_naive.py``  (``iso_kdn_gain_naive``,
  ``_memory_recurrence``, ``naive_recurrent_iso_kdn``, ``_naive_chunk_iso_kdn``)
* ``lit_gpt/kdn_ops/diag_kdn_naive.py`` (``diag_kdn_gain_naive``,
  ``_memory_recurrence``, ``naive_recurrent_diag_kdn``, ``_naive_chunk_diag_kdn``)

They are loaded by file path (the package ``__init__`` needs Lightning), run in
float64 on seeded inputs, and their outputs and autograd gradients are written
to ``tests/golden/*.npz``.  Usage::

    python tests/golden/make_golden.py --reference <checkout of ngocbh/kalman-delta-networks>

The fixtures are committed; this script is only re-run when a case is added.
"""
from __future__ import annotations

import argparse
import importlib.util
import math
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LN2 = math.log(2.0)


def _load(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def _l2norm(x, eps=1e-6):
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def _alpha_from_G(G, chunk):
    T = G.shape[1]
    prev = torch.zeros_like(G)
    prev[:, 1:] = G[:, :-1]
    starts = (torch.arange(T) % chunk == 0).view(1, T, 1, 1)
    prev = torch.where(starts, torch.zeros_like(G), prev)
    return torch.exp(G - prev)


def _g_cumsum(log_alpha, chunk):
    out = torch.empty_like(log_alpha)
    for s in range(0, log_alpha.shape[1], chunk):
        out[:, s:s + chunk] = log_alpha[:, s:s + chunk].cumsum(1) / LN2
    return out


def case_iso_gain(iso, gen):
    """iso_kdn_gain_naive with unit keys and alpha = sqrt(a) in every channel,
    so mean(alpha^2) = a and ||k||^2 = 1: the production ``iso_kdn_gain`` inputs."""
    B, T, H, K = 2, 150, 3, 8
    a = torch.rand(B, T, H, generator=gen).float() * 0.98 + 0.01
    omega = torch.nn.functional.softplus(torch.randn(B, T, H, generator=gen)).float()
    r = (0.01 + torch.nn.functional.softplus(torch.randn(B, T, H, generator=gen))).float()
    prec = (0.1 + torch.nn.functional.softplus(torch.randn(H, generator=gen))).float()
    dbeta = torch.randn(B, T, H, generator=gen).float()
    out = {"a": a, "omega": omega, "r": r, "initial_precision": prec, "dbeta": dbeta}
    for tag, info_scale in (("s1", float(K)), ("s05", 0.5 * K)):
        la, lw, lr, lp = (t.double().clone().requires_grad_(True) for t in (a, omega, r, prec))
        k = torch.zeros(B, T, H, K, dtype=torch.float64)
        k[..., 0] = 1.0
        alpha = la.sqrt()[..., None].expand(B, T, H, K)
        beta, final_precision = iso.iso_kdn_gain_naive(
            k, alpha, lw, lr, info_scale=info_scale, initial_precision=lp, output_final_state=True
        )
        (beta * dbeta.double()).sum().backward()
        out[f"{tag}_posterior_scale"] = torch.tensor(info_scale / K)
        out[f"{tag}_beta"] = beta
        out[f"{tag}_final_precision"] = final_precision
        out[f"{tag}_da"], out[f"{tag}_domega"] = la.grad, lw.grad
        out[f"{tag}_dr"], out[f"{tag}_dprec"] = lr.grad, lp.grad
    return out


def case_diag_gain(diag, gen):
    B, T, H, K = 2, 70, 2, 16
    k = torch.randn(B, T, H, K, generator=gen).float()
    alpha = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, H, K, generator=gen))).float()
    omega = torch.nn.functional.softplus(torch.randn(B, T, H, K, generator=gen)).float()
    r = (0.01 + torch.nn.functional.softplus(torch.randn(B, T, H, generator=gen))).float()
    prec = (0.1 + torch.nn.functional.softplus(torch.randn(H, generator=gen))).float()
    dkappa = torch.randn(B, T, H, K, generator=gen).float()
    lk, la, lw, lr, lp = (t.double().clone().requires_grad_(True) for t in (k, alpha, omega, r, prec))
    kappa, final_precision = diag.diag_kdn_gain_naive(lk, la, lw, lr, initial_precision=lp, output_final_state=True)
    (kappa * dkappa.double()).sum().backward()
    chunk_kappa, chunk_prec = diag._chunk_diag_kdn_gain(
        k.double(), alpha.double(), omega.double(), r.double(), initial_precision=prec.double(),
        output_final_state=True, chunk_size=32,
    )
    assert torch.allclose(chunk_kappa, kappa.detach(), rtol=1e-9, atol=1e-12)
    assert torch.allclose(chunk_prec, final_precision.detach(), rtol=1e-9, atol=1e-12)
    return {
        "k": k, "alpha": alpha, "omega": omega, "r": r, "initial_precision": prec, "dkappa": dkappa,
        "kappa": kappa, "final_precision": final_precision, "dk": lk.grad, "dalpha": la.grad,
        "domega": lw.grad, "dr": lr.grad, "dprec": lp.grad,
    }


def case_memory(mod, gen, tag):
    """The reference ``_memory_recurrence`` with a non-zero initial memory."""
    B, T, H, K, V = 1, 70, 2, 16, 8
    q = torch.randn(B, T, H, K, generator=gen).float()
    k = _l2norm(torch.randn(B, T, H, K, generator=gen)).float()
    v = torch.randn(B, T, H, V, generator=gen).float()
    alpha = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, H, K, generator=gen))).float()
    if tag == "iso":
        gain = torch.sigmoid(torch.randn(B, T, H, generator=gen)).float()
    else:
        gain = (0.2 * torch.randn(B, T, H, K, generator=gen)).float()
    S0 = torch.randn(B, H, K, V, generator=gen).float()
    dO = torch.randn(B, T, H, V, generator=gen).float()
    dS = torch.randn(B, H, K, V, generator=gen).float()
    leaves = [t.double().clone().requires_grad_(True) for t in (q, k, v, alpha, gain, S0)]
    o, S = mod._memory_recurrence(*leaves, 0.3)
    ((o * dO.double()).sum() + (S * dS.double()).sum()).backward()
    names = ("q", "k", "v", "alpha", "gain", "S0")
    out = {n: t for n, t in zip(names, (q, k, v, alpha, gain, S0))}
    out.update({"dO": dO, "dS": dS, "o": o, "S": S})
    out.update({"d" + n: leaf.grad for n, leaf in zip(names, leaves)})
    return out


def case_iso_scan(iso, gen):
    """Semantics of ``_chunk_kda_precumsum_paired``: l2norm(q, k), kappa = beta*k_hat,
    alpha from the 64-local base-2 g_cumsum, reference ``_memory_recurrence``.
    T=130 spans two full 64-chunks and a 2-token tail."""
    B, T, H, K, V = 1, 130, 2, 32, 32
    q = torch.randn(B, T, H, K, generator=gen).bfloat16().float()
    k = torch.randn(B, T, H, K, generator=gen).bfloat16().float()
    v = torch.randn(B, T, H, V, generator=gen).bfloat16().float()
    log_alpha = -torch.nn.functional.softplus(torch.randn(B, T, H, K, generator=gen))
    g = _g_cumsum(log_alpha, 64).float()
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen)).float()
    dO = torch.randn(B, T, H, V, generator=gen).bfloat16().float()
    lq, lk, lv, lb = (t.double().clone().requires_grad_(True) for t in (q, k, v, beta))
    G = (g.double() * LN2).requires_grad_(True)
    qh, kh = _l2norm(lq), _l2norm(lk)
    o, S = iso._memory_recurrence(qh, kh, lv, _alpha_from_G(G, 64), lb, torch.zeros(B, H, K, V, dtype=torch.float64), K ** -0.5)
    (o * dO.double()).sum().backward()
    return {"q": q, "k": k, "v": v, "g_cumsum": g, "beta": beta, "dO": dO, "o": o, "S": S,
            "dq": lq.grad, "dk": lk.grad, "dv": lv.grad, "dg": G.grad, "dbeta": lb.grad}


def case_diag_scan(diag, gen):
    """Semantics of ``chunk_kalman``: alpha from the 32-local g_cumsum, kappa the
    write vector, reference ``_memory_recurrence``.  T=70: two 32-chunks + 6."""
    B, T, H, K, V = 1, 70, 2, 32, 32
    q = _l2norm(torch.randn(B, T, H, K, generator=gen)).bfloat16().float()
    k = _l2norm(torch.randn(B, T, H, K, generator=gen)).bfloat16().float()
    v = torch.randn(B, T, H, V, generator=gen).bfloat16().float()
    log_alpha = -torch.nn.functional.softplus(torch.randn(B, T, H, K, generator=gen))
    g = _g_cumsum(log_alpha, 32).float()
    kappa = (0.3 * torch.randn(B, T, H, K, generator=gen)).float()
    dO = torch.randn(B, T, H, V, generator=gen).float()
    lq, lk, lkap, lv = (t.double().clone().requires_grad_(True) for t in (q, k, kappa, v))
    G = (g.double() * LN2).requires_grad_(True)
    o, S = diag._memory_recurrence(lq, lk, lv, _alpha_from_G(G, 32), lkap, torch.zeros(B, H, K, V, dtype=torch.float64), K ** -0.5)
    (o * dO.double()).sum().backward()
    return {"q": q, "k": k, "kappa": kappa, "v": v, "g_cumsum": g, "dO": dO, "o": o, "S": S,
            "dq": lq.grad, "dk": lk.grad, "dkappa": lkap.grad, "dv": lv.grad, "dg": G.grad}


def case_full(iso, diag, gen):
    """Config-0 style end-to-end oracles (gain + memory) at a reduced width, and
    the reference's private chunked oracles checked against them."""
    B, T, H, K, V = 1, 100, 2, 16, 16
    q = _l2norm(torch.randn(B, T, H, K, generator=gen)).float()
    k = _l2norm(torch.randn(B, T, H, K, generator=gen)).float()
    v = torch.randn(B, T, H, V, generator=gen).float()
    alpha = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, H, K, generator=gen))).float()
    omega_s = torch.nn.functional.softplus(torch.randn(B, T, H, generator=gen)).float()
    omega_v = torch.nn.functional.softplus(torch.randn(B, T, H, K, generator=gen)).float()
    r = (0.01 + torch.nn.functional.softplus(torch.randn(B, T, H, generator=gen))).float()
    args = (q.double(), k.double(), v.double(), alpha.double())
    o_iso, (S_iso, p_iso) = iso.naive_recurrent_iso_kdn(*args, omega_s.double(), r.double(), output_final_state=True)
    o_isoc, (S_isoc, p_isoc) = iso._naive_chunk_iso_kdn(*args, omega_s.double(), r.double(), output_final_state=True)
    o_dg, (S_dg, p_dg) = diag.naive_recurrent_diag_kdn(*args, omega_v.double(), r.double(), output_final_state=True)
    o_dgc, (S_dgc, p_dgc) = diag._naive_chunk_diag_kdn(*args, omega_v.double(), r.double(), output_final_state=True)
    for x, y in ((o_iso, o_isoc), (S_iso, S_isoc), (p_iso, p_isoc), (o_dg, o_dgc), (S_dg, S_dgc), (p_dg, p_dgc)):
        assert torch.allclose(x, y, rtol=1e-8, atol=1e-10), (x - y).abs().max()
    return {"q": q, "k": k, "v": v, "alpha": alpha, "omega_s": omega_s, "omega_v": omega_v, "r": r,
            "iso_o": o_iso, "iso_S": S_iso, "iso_precision": p_iso,
            "diag_o": o_dg, "diag_S": S_dg, "diag_precision": p_dg}


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("KDN_REFERENCE_ROOT"), required=False)
    args = parser.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <reference checkout> or set KDN_REFERENCE_ROOT")
    ops = os.path.join(args.reference, "lit_gpt", "kdn_ops")
    iso = _load(os.path.join(ops, "iso_kdn_naive.py"), "ref_iso_kdn_naive")
    diag = _load(os.path.join(ops, "diag_kdn_naive.py"), "ref_diag_kdn_naive")
    torch.set_num_threads(4)
    cases = {
        "iso_gain": lambda g: case_iso_gain(iso, g),
        "diag_gain": lambda g: case_diag_gain(diag, g),
        "iso_memory": lambda g: case_memory(iso, g, "iso"),
        "diag_memory": lambda g: case_memory(diag, g, "diag"),
        "iso_scan": lambda g: case_iso_scan(iso, g),
        "diag_scan": lambda g: case_diag_scan(diag, g),
        "full": lambda g: case_full(iso, diag, g),
    }
    for seed, (name, fn) in enumerate(cases.items()):
        gen = torch.Generator().manual_seed(1000 + seed)
        data = fn(gen)
        arrays = {}
        for key, value in data.items():
            value = value.detach()
            arrays[key] = _np(value.float() if value.dtype == torch.float32 else value)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **arrays)
        print(f"{name}: {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
