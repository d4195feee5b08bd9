"""Generate ``tests/golden/iso_gate.npz`` and ``tests/golden/diag_gate.npz``:
the reference's own gate frontends evaluated on seeded inputs, the isotropic
one (``_iso_kdn_gate_precumsum_fwd`` / ``_bwd``,
lit_gpt/kdn_ops/iso_kdn_chunk.py:1059-1314) and the diagonal one
(``_diag_kdn_frontend_forward`` / ``_backward``,
lit_gpt/kdn_ops/diag_kdn_chunk.py:2218-2443).

The reference implements the frontends only as Triton kernels, and there is no
PyTorch oracle for them; they run here on the CPU under Triton's interpreter
(``TRITON_INTERPRET=1``), where flash-linear-attention selects its plain
Triton softplus (x above 20, else ln(1 + e^x)) instead of the inline-PTX one.
Usage::

    python tests/golden/make_gate_golden.py --reference <checkout of ngocbh/kalman-delta-networks>

The fixture is committed; this script is only re-run when a case is added.
"""
from __future__ import annotations

import argparse
import contextlib
import importlib.util
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402

# (B, T, H, K, g_raw bf16, omega_r_raw bf16, omega_min, r_min, seed)
CASES = [
    (1, 70, 2, 64, False, False, 1e-3, 1e-2, 11),
    (2, 80, 2, 128, True, True, 0.0, 0.01, 12),
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    path = os.path.join(args.reference, "lit_gpt", "kdn_ops", "iso_kdn_chunk.py")
    spec = importlib.util.spec_from_file_location("ref_iso_kdn_chunk", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    torch.cuda.device = lambda device: contextlib.nullcontext()  # CPU tensors under the interpreter
    out = {}
    for ci, (B, T, H, K, gbf, wbf, wmin, rmin, seed) in enumerate(CASES):
        inputs, cot = oracle.make_iso_gate_inputs(B, T, H, K, seed=seed,
                                                  g_dtype=torch.bfloat16 if gbf else torch.float32,
                                                  wr_dtype=torch.bfloat16 if wbf else torch.float32)
        fwd = ref._iso_kdn_gate_precumsum_fwd(*inputs, wmin, rmin)
        a = fwd[1]
        grads = ref._iso_kdn_gate_precumsum_bwd(*inputs, a, *cot, (True,) * 7)
        p = f"c{ci}_"
        out[p + "meta"] = np.array([B, T, H, K, int(gbf), int(wbf), wmin, rmin], dtype=np.float64)
        for n, t in zip(("g_raw", "omega_r_raw", "omega_bias", "r_bias", "A_log", "dt_bias", "param"), inputs):
            out[p + n] = t.float().numpy()
        for n, t in zip(("dg_pre", "da", "domega", "dr", "dinit"), cot):
            out[p + n] = t.float().numpy()
        for n, t in zip(("g_cumsum", "a", "omega", "r", "initial_precision"), fwd):
            out[p + n] = t.float().numpy()
        for n, t in zip(("dg_raw", "domega_r_raw", "domega_bias", "dr_bias", "dA_log", "ddt_bias", "dparam"), grads):
            out[p + n] = t.float().numpy()
    np.savez_compressed(os.path.join(HERE, "iso_gate.npz"), **out)
    print("wrote", os.path.join(HERE, "iso_gate.npz"), len(CASES), "cases")
    diag_golden(args.reference)


# (B, T, H, K, seed): T not a multiple of the 32-token chunk
DIAG_CASES = [
    (1, 45, 2, 64, 21),
    (2, 36, 1, 128, 22),
]


def diag_golden(reference):
    path = os.path.join(reference, "lit_gpt", "kdn_ops", "diag_kdn_chunk.py")
    spec = importlib.util.spec_from_file_location("ref_diag_kdn_chunk", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    out = {}
    for ci, (B, T, H, K, seed) in enumerate(DIAG_CASES):
        inputs, cot = oracle.make_diag_gate_inputs(B, T, H, K, seed=seed)
        fwd = ref._diag_kdn_frontend_forward(*inputs)
        grads = ref._diag_kdn_frontend_backward(*inputs, fwd[1], *cot, (True,) * 6)
        p = f"c{ci}_"
        out[p + "meta"] = np.array([B, T, H, K], dtype=np.int64)
        for n, t in zip(DIAG_INPUTS, inputs):
            out[p + n] = t.float().numpy()
        for n, t in zip(DIAG_COTANGENTS, cot):
            out[p + n] = t.float().numpy()
        for n, t in zip(DIAG_OUTPUTS, fwd):
            out[p + n] = t.float().numpy()
        for n, t in zip(DIAG_GRADS, grads):
            out[p + n] = t.float().numpy()
    np.savez_compressed(os.path.join(HERE, "diag_gate.npz"), **out)
    print("wrote", os.path.join(HERE, "diag_gate.npz"), len(DIAG_CASES), "cases")


DIAG_INPUTS = ("retention_raw", "omega_raw", "r_raw", "A_log", "dt_bias", "param")
DIAG_COTANGENTS = ("d_g_cumsum", "d_alpha", "d_omega", "d_r", "d_init")
DIAG_OUTPUTS = ("g_cumsum", "alpha", "omega", "r", "initial_precision")
DIAG_GRADS = ("dretention_raw", "domega_raw", "dr_raw", "dA_log", "ddt_bias", "dparam")


if __name__ == "__main__":
    main()
