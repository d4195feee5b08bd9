"""ctypes binding of ``libkdn_b200.so`` (C ABI in ``include/kdn_b200.h``).

The shared library is required: importing the operators works without a GPU,
but every call raises ``RuntimeError`` when the library or a CUDA device is
missing.  There is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("KDN_B200_LIB", os.path.join(_HERE, "lib", "libkdn_b200.so"))

KDN_OK = 0
KDN_ISO = 0
KDN_DIAG = 1
KDN_PREC_BF16 = 0
KDN_PREC_FP32 = 1
# passes of a scan call (KdnScanArgs.mode)
KDN_SCAN_FULL = 0
KDN_SCAN_FWD_RECORDS = 1
KDN_SCAN_FWD_SEQUENTIAL = 2
KDN_SCAN_FWD_STATE_MAP = 3
KDN_SCAN_BWD_STATE = 4

_lock = threading.Lock()
_lib = None


class KdnScanArgs(ctypes.Structure):
    _fields_ = [
        ("variant", ctypes.c_int32),
        ("precision", ctypes.c_int32),
        ("B", ctypes.c_int64),
        ("T", ctypes.c_int64),
        ("H", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("V", ctypes.c_int64),
        ("scale", ctypes.c_float),
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("g", ctypes.c_void_p),
        ("beta", ctypes.c_void_p),
        ("kappa", ctypes.c_void_p),
        ("initial_state", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("final_state", ctypes.c_void_p),
        ("saved", ctypes.c_void_p),
        ("dO", ctypes.c_void_p),
        ("d_final_state", ctypes.c_void_p),
        ("dq", ctypes.c_void_p),
        ("dk", ctypes.c_void_p),
        ("dv", ctypes.c_void_p),
        ("dg", ctypes.c_void_p),
        ("dbeta", ctypes.c_void_p),
        ("dkappa", ctypes.c_void_p),
        ("d_initial_state", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("mode", ctypes.c_int32),
        ("final_state_map", ctypes.c_void_p),
        ("varlen_table", ctypes.c_void_p),
        ("num_seqs", ctypes.c_int64),
        ("num_chunks", ctypes.c_int64),
    ]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_F = ctypes.c_float
_SZ = ctypes.c_size_t

_SIGNATURES = {
    "kdn_version": ([], ctypes.c_int),
    "kdn_last_error": ([], ctypes.c_char_p),
    "kdn_iso_gain_workspace_bytes": ([_I64, _I64, _I64], _SZ),
    "kdn_iso_gain_fwd": ([_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _F, _P, _SZ, _P], ctypes.c_int),
    "kdn_iso_gain_bwd": (
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _F, _P, _SZ, _P],
        ctypes.c_int,
    ),
    "kdn_iso_gain_fwd_maps": ([_P, _P, _P, _P, _I64, _I64, _I64, _F, _P, _SZ, _P], ctypes.c_int),
    "kdn_iso_gain_fwd_finish": ([_P] * 8 + [_I64, _I64, _I64, _F, _P, _SZ, _P], ctypes.c_int),
    "kdn_iso_gain_bwd_maps": ([_P] * 6 + [_I64, _I64, _I64, _F, _P, _SZ, _P], ctypes.c_int),
    "kdn_iso_gain_bwd_finish": ([_P] * 13 + [_I64, _I64, _I64, _F, _P, _SZ, _P], ctypes.c_int),
    "kdn_iso_gain_varlen_workspace_bytes": ([_I64, _I64, _I64], _SZ),
    "kdn_iso_gain_fwd_varlen": ([_P] * 8 + [_I64, _I64, _F, _P, _I64, _I64, _P, _SZ, _P], ctypes.c_int),
    "kdn_iso_gain_bwd_varlen": ([_P] * 13 + [_I64, _I64, _F, _P, _I64, _I64, _P, _SZ, _P], ctypes.c_int),
    "kdn_iso_gate_workspace_bytes": ([_I64, _I64, _I64, _I64], _SZ),
    "kdn_iso_gate_fwd": (
        [_P, ctypes.c_int, _P, ctypes.c_int, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
         _I64, _I64, _I64, _I64, _F, _F, _P],
        ctypes.c_int,
    ),
    "kdn_iso_gate_bwd": (
        [_P, ctypes.c_int, _P, ctypes.c_int, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
         _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _SZ, _P],
        ctypes.c_int,
    ),
    "kdn_diag_gate_workspace_bytes": ([_I64, _I64, _I64, _I64], _SZ),
    "kdn_diag_gate_fwd": ([_P] * 11 + [_I64, _I64, _I64, _I64, _P], ctypes.c_int),
    "kdn_diag_gate_bwd": ([_P] * 17 + [_I64, _I64, _I64, _I64, _P, _SZ, _P], ctypes.c_int),
    "kdn_diag_gain_carry_elems": ([_I64, _I64, _I64, _I64], _I64),
    "kdn_diag_gain_workspace_bytes": ([_I64, _I64, _I64, _I64], _SZ),
    "kdn_diag_gain_fwd": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _SZ, _P], ctypes.c_int),
    "kdn_diag_gain_fwd_noalloc": ([_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P], ctypes.c_int),
    "kdn_diag_gain_fwd_maps": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _SZ, _P], ctypes.c_int),
    "kdn_diag_gain_fwd_finish": ([_P] * 9 + [_I64, _I64, _I64, _I64, _P, _SZ, _P], ctypes.c_int),
    "kdn_diag_gain_bwd_maps": ([_P] * 7 + [_I64, _I64, _I64, _I64, _P, _SZ, _P], ctypes.c_int),
    "kdn_diag_gain_bwd_finish": ([_P] * 17 + [_I64, _I64, _I64, _I64, _P, _SZ, _P], ctypes.c_int),
    "kdn_diag_gain_bwd": (
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _SZ, _P],
        ctypes.c_int,
    ),
    "kdn_diag_gain_varlen_carry_elems": ([_I64, _I64, _I64, _I64], _I64),
    "kdn_diag_gain_varlen_workspace_bytes": ([_I64, _I64, _I64, _I64], _SZ),
    "kdn_diag_gain_fwd_varlen": ([_P] * 9 + [_I64, _I64, _I64, _P, _I64, _I64, _P, _SZ, _P], ctypes.c_int),
    "kdn_diag_gain_bwd_varlen": ([_P] * 17 + [_I64, _I64, _I64, _P, _I64, _I64, _P, _SZ, _P], ctypes.c_int),
    "kdn_varlen_table_len": ([_I64, _I64], _I64),
    "kdn_varlen_plan": ([_P, _I64, _P, _I64, ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "kdn_diag_norm_fwd": ([_P, _P, ctypes.c_int, _P, _P, _P, _P, _P, _I64, _I64, _P], ctypes.c_int),
    "kdn_diag_norm_bwd": ([_P, _P, ctypes.c_int, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _P], ctypes.c_int),
    "kdn_rmsnorm_gated_workspace_bytes": ([_I64, _I64], _SZ),
    "kdn_rmsnorm_gated_fwd": ([_P, ctypes.c_int, _P, ctypes.c_int, _P, _P, _P, _I64, _I64, _F, ctypes.c_int, _P],
                              ctypes.c_int),
    "kdn_rmsnorm_gated_bwd": ([_P, ctypes.c_int, _P, ctypes.c_int, _P, _P, _P, _P, _P, _P, _I64, _I64, ctypes.c_int,
                               _P, _SZ, _P], ctypes.c_int),
    "kdn_short_conv_workspace_bytes": ([_I64, _I64, _I64, _I64], _SZ),
    "kdn_short_conv_fwd": ([_P, ctypes.c_int, _P, ctypes.c_int, _P, _I64, _I64, _I64, _I64, _I64, ctypes.c_int, _P],
                           ctypes.c_int),
    "kdn_short_conv_bwd": ([_P, ctypes.c_int, _P, ctypes.c_int, _P, _I64, _P, _P, _I64, _I64, _I64, _I64,
                            ctypes.c_int, _P, _SZ, _P], ctypes.c_int),
    "kdn_scan_saved_bytes": ([ctypes.POINTER(KdnScanArgs)], _SZ),
    "kdn_scan_workspace_bytes": ([ctypes.POINTER(KdnScanArgs)], _SZ),
    "kdn_scan_fwd": ([ctypes.POINTER(KdnScanArgs), _P], ctypes.c_int),
    "kdn_scan_bwd": ([ctypes.POINTER(KdnScanArgs), _P], ctypes.c_int),
}


def load_library():
    """Load the C-ABI library once; raise a clear error when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"kdn_b200: native library not found at {LIB_PATH}; build it with "
                    "`python -m kdn_b200.build` (nvcc, sm_100a)"
                )
            lib = ctypes.CDLL(LIB_PATH)
            for name, (argtypes, restype) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = restype
            _lib = lib
    return _lib


def exported_symbols():
    return tuple(_SIGNATURES)


def check(rc: int, what: str) -> None:
    if rc != KDN_OK:
        msg = load_library().kdn_last_error().decode(errors="replace")
        raise RuntimeError(f"kdn_b200 {what} failed ({rc}): {msg}")


def require_cuda(*tensors: torch.Tensor) -> None:
    if not torch.cuda.is_available():
        raise RuntimeError("kdn_b200 kernels need a CUDA device (B200, sm_100a); there is no CPU fallback")
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("kdn_b200 kernels need CUDA tensors")
    load_library()


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


_PRECISION = {"bf16": KDN_PREC_BF16, "fp32": KDN_PREC_FP32}


def precision() -> int:
    """Arithmetic precision of the scan, chosen by ``KDN_B200_PRECISION``:
    "bf16" (the product: the tcgen05 tensor-core kernels with bf16 operands
    and fp32 accumulation) or "fp32" (a separate debug implementation of the
    same chunked algorithm: SIMT / fp32 kernels with fp32 operands and the
    diagonal scan on 32-token chunks, used as a tight cross-check of the
    algorithm, not of the tcgen05 kernels)."""
    name = os.environ.get("KDN_B200_PRECISION", "bf16").lower()
    if name not in _PRECISION:
        raise ValueError(f"KDN_B200_PRECISION must be one of {sorted(_PRECISION)}, got {name!r}")
    return _PRECISION[name]


def byte_buffer(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)
