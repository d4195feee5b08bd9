"""Generate ``tests/golden/diag_norm.npz``: the reference's own diagonal q / k
normalisation (``_diag_kdn_normalize``, lit_gpt/kdn_ops/diag_kdn_chunk.py:2162,
kernels :194 and :235), forward and backward, on seeded inputs.

Its kernels are Triton with inline PTX (``div.rn``, ``sqrt.rn``, warp
shuffles), which Triton's CPU interpreter cannot run, so this script runs
them on a GPU, through the reference's stock entry point and autograd
Function, from an unmodified install of the reference (``baseline/_ref`` by
default, ``--reference`` for another checkout).  Usage, on a machine with a
CUDA device::

    python tests/golden/make_norm_golden.py [--reference <checkout>] [--out tests/golden/diag_norm.npz]

The cases cover the reduction orders the reference switches between (calls of
>= 16, 8-15 and < 8 rows), K = 64 and 128, bf16 and fp32 inputs, rows of zeros
and every subset of cotangents the backward distinguishes.  The fixture is
committed; the script is only re-run when a case is added.
"""
from __future__ import annotations

import argparse
import importlib.util
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

# name: (B, T, H, K, dtype, cotangents present (q_memory, k_gain, k_memory), seed)
CASES = {
    "rows222": (2, 37, 3, 128, torch.bfloat16, (True, True, True), 1),
    "rows12": (1, 4, 3, 128, torch.bfloat16, (True, False, True), 2),
    "rows5": (1, 5, 1, 128, torch.bfloat16, (False, True, False), 3),
    "k64_rows80": (2, 20, 2, 64, torch.bfloat16, (True, True, True), 4),
    "k64_rows6": (1, 3, 2, 64, torch.bfloat16, (True, True, False), 5),
    "fp32_rows18": (1, 9, 2, 128, torch.float32, (True, True, True), 6),
}


def make_case(B, T, H, K, dtype, present, seed, device):
    gen = torch.Generator().manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=gen)  # noqa: E731
    # row magnitudes over 2^-8 .. 2^8 exercise the rounding of every step
    scale = torch.exp2(torch.randint(-8, 9, (B, T, H, 1), generator=gen).float())
    q = (n(B, T, H, K) * scale).to(dtype)
    k = (n(B, T, H, K) * scale.flip(1)).to(dtype)
    q.view(-1, K)[0] = 0  # a row of zeros (norm 0)
    k.view(-1, K)[-1] = 0
    cots = (n(B, T, H, K).bfloat16(), n(B, T, H, K), n(B, T, H, K).bfloat16())
    cots = tuple(c.to(device) if p else None for c, p in zip(cots, present))
    return q.to(device), k.to(device), cots


def bits(t):
    t = t.detach().cpu()
    return t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.path.join(ROOT, "baseline", "_ref"))
    ap.add_argument("--out", default=os.path.join(HERE, "diag_norm.npz"))
    args = ap.parse_args()
    path = os.path.join(args.reference, "lit_gpt", "kdn_ops", "diag_kdn_chunk.py")
    spec = importlib.util.spec_from_file_location("ref_diag_kdn_chunk", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    dev = torch.device("cuda")
    out = {}
    for name, (B, T, H, K, dtype, present, seed) in CASES.items():
        q, k, cots = make_case(B, T, H, K, dtype, present, seed, dev)
        ql, kl = q.clone().requires_grad_(True), k.clone().requires_grad_(True)
        q_memory, k_gain, k_memory = ref._diag_kdn_normalize(ql, kl)
        used = [(o, c) for o, c in zip((q_memory, k_gain, k_memory), cots) if c is not None]
        torch.autograd.backward([o for o, _ in used], [c for _, c in used])
        p = name + "_"
        out[p + "meta"] = np.array([B, T, H, K, int(dtype == torch.bfloat16), *present], dtype=np.int64)
        for key, t in (("q", q), ("k", k), ("q_memory", q_memory), ("k_gain", k_gain), ("k_memory", k_memory),
                       ("dq", ql.grad), ("dk", kl.grad)):
            if t is not None:
                out[p + key] = bits(t)
        for key, c in zip(("d_q_memory", "d_k_gain", "d_k_memory"), cots):
            if c is not None:
                out[p + key] = bits(c)
    np.savez_compressed(args.out, **out)
    print("wrote", args.out, sorted({k.split("_")[0] for k in out}))


if __name__ == "__main__":
    main()
