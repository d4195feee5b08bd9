"""Generate ``tests/golden/norm_gated.npz``: flash-linear-attention's own
gated RMS normalisation (``fla.modules.fused_norm_gate.rms_norm_gated``, the
``FusedRMSNormGated`` the reference mixers apply to the scan output,
lit_gpt/iso_kdn.py:192-197 and diag_kdn.py:216-221), forward and backward,
on seeded inputs.

Its kernels are plain Triton, so they run here on the CPU under Triton's
interpreter (``TRITON_INTERPRET=1``).  The installed flash-linear-attention
is 0.5.1; the reference pins commit 4b02d15d6a68700181b180235be62a9fb95d2a38,
whose gated norm computes the same published formula.  Usage::

    python tests/golden/make_norm_gated_golden.py

The fixture is committed; the script is only re-run when a case is added.
"""
from __future__ import annotations

import contextlib
import os

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (rows shape, D, x dtype, g dtype, activation, with weight, seed)
CASES = {
    "sigmoid_bf16": ((2, 40, 3), 128, torch.bfloat16, torch.bfloat16, "sigmoid", True, 1),
    "swish_fp32": ((1, 33, 2), 64, torch.float32, torch.float32, "swish", True, 2),
    "sigmoid_noweight": ((3, 17), 128, torch.float32, torch.bfloat16, "sigmoid", False, 3),
}


def main():
    # CPU tensors under the interpreter: no device context (flash-linear-attention
    # picks torch.cpu as its device library when no GPU is present)
    torch.cuda.device = lambda device: contextlib.nullcontext()
    torch.cpu.device = lambda device: contextlib.nullcontext()
    # the interpreter has no device to time autotuning candidates on; every
    # candidate differs only in num_warps, so score them all equal (the first runs)
    import triton.runtime.autotuner as autotuner

    autotuner.Autotuner._bench = lambda self, *args, config, **meta: [1.0, 1.0, 1.0]
    import fla.modules.fused_norm_gate as fng

    # the backward splits its weight-gradient partial sums over the device's
    # SMs; the interpreter has no device, so give it a B200's 148
    fng.get_multiprocessor_count = lambda *args, **kwargs: 148
    rms_norm_gated = fng.rms_norm_gated

    out = {}
    for name, (shape, D, xdt, gdt, act, has_w, seed) in CASES.items():
        gen = torch.Generator().manual_seed(seed)
        x = (torch.randn(*shape, D, generator=gen) * 2.0).to(xdt)
        g = torch.randn(*shape, D, generator=gen).to(gdt)
        w = (1.0 + 0.3 * torch.randn(D, generator=gen)) if has_w else None
        dy = torch.randn(*shape, D, generator=gen).to(xdt)
        xl, gl = x.clone().requires_grad_(True), g.clone().requires_grad_(True)
        wl = w.clone().requires_grad_(True) if has_w else None
        y = rms_norm_gated(xl, gl, wl, None, act, eps=1e-5)
        y.backward(dy)
        p = name + "_"
        out[p + "meta"] = np.array([D, int(xdt == torch.bfloat16), int(gdt == torch.bfloat16),
                                    int(act == "swish"), int(has_w)], dtype=np.int64)
        for key, t in (("x", x), ("g", g), ("w", w), ("dy", dy), ("y", y), ("dx", xl.grad), ("dg", gl.grad),
                       ("dw", None if wl is None else wl.grad)):
            if t is not None:
                t = t.detach()
                out[p + key] = t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()
    np.savez_compressed(os.path.join(HERE, "norm_gated.npz"), **out)
    print("wrote", os.path.join(HERE, "norm_gated.npz"), sorted(CASES))


if __name__ == "__main__":
    main()
