"""Generate ``tests/golden/short_conv.npz``: the reference's own packed q/k/v
short convolution (``qkv_causal_conv1d``, lit_gpt/kdn_ops/iso_kdn_chunk.py:459:
flash-linear-attention's causal_conv1d forward and the reference's grouped
backward kernel), forward and backward, on seeded inputs.

Both are plain Triton, so they run on the CPU under Triton's interpreter
(``TRITON_INTERPRET=1``), from an unmodified install of the reference
(``baseline/_ref`` by default, ``--reference`` for another checkout)::

    python tests/golden/make_conv_golden.py [--reference <checkout>]

The fixture is committed; the script is only re-run when a case is added.
"""
from __future__ import annotations

import argparse
import contextlib
import importlib.util
import os

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

# name: (B, T, D, x dtype, weight dtype, seed)
CASES = {
    "bf16_T70": (2, 70, 64, torch.bfloat16, torch.float32, 1),
    "fp32_T5": (1, 5, 32, torch.float32, torch.float32, 2),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.path.join(ROOT, "baseline", "_ref"))
    args = ap.parse_args()
    # CPU tensors under the interpreter: no device context, no timing of
    # autotuning candidates, a B200's SM count where the code asks for one
    torch.cuda.device = lambda device: contextlib.nullcontext()
    torch.cpu.device = lambda device: contextlib.nullcontext()
    import triton.runtime.autotuner as autotuner

    autotuner.Autotuner._bench = lambda self, *a, config, **meta: [1.0, 1.0, 1.0]
    path = os.path.join(args.reference, "lit_gpt", "kdn_ops", "iso_kdn_chunk.py")
    spec = importlib.util.spec_from_file_location("ref_iso_kdn_chunk", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    out = {}
    for name, (B, T, D, xdt, wdt, seed) in CASES.items():
        gen = torch.Generator().manual_seed(seed)
        x = torch.randn(B, T, 3 * D, generator=gen).to(xdt)
        w = (torch.randn(3 * D, 4, generator=gen) * 0.5).to(wdt)
        dys = [torch.randn(B, T, D, generator=gen).to(xdt) for _ in range(3)]
        xl, wl = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
        # the interpreter runs on CPU tensors; the reference's validation wants "cuda"
        ref._validate_qkv_conv_inputs = lambda a, b: a.shape[-1] // 3
        q, k, v = ref._QKVCausalConv1d.apply(xl, wl)
        torch.autograd.backward([q, k, v], dys)
        p = name + "_"
        out[p + "meta"] = np.array([B, T, D, int(xdt == torch.bfloat16), int(wdt == torch.bfloat16)], dtype=np.int64)
        for key, t in (("x", x), ("w", w), ("dq", dys[0]), ("dk", dys[1]), ("dv", dys[2]), ("q", q), ("k", k),
                       ("v", v), ("dx", xl.grad), ("dw", wl.grad)):
            t = t.detach()
            out[p + key] = t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()
    np.savez_compressed(os.path.join(HERE, "short_conv.npz"), **out)
    print("wrote", os.path.join(HERE, "short_conv.npz"), sorted(CASES))


if __name__ == "__main__":
    main()
