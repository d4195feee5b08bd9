"""CPU checks of the C-ABI library: it loads, exports every symbol the public
header declares, and the host-side size queries and argument validation
work without a GPU (no kernel is launched)."""
import ctypes
import os
import re

import pytest

from kdn_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kdn_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const char\*|size_t|int64_t|int)\s+(kdn_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(N.LIB_PATH):
        from kdn_b200 import build

        build.build()
    return N.load_library()


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for required in ("kdn_scan_fwd", "kdn_scan_bwd", "kdn_iso_gain_fwd", "kdn_iso_gain_bwd",
                     "kdn_diag_gain_fwd", "kdn_diag_gain_bwd", "kdn_last_error", "kdn_version"):
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(N.exported_symbols()) >= set(declared_functions())


def test_version(lib):
    assert lib.kdn_version() == 102


def test_scan_size_queries(lib):
    a = N.KdnScanArgs()
    a.variant, a.precision = N.KDN_ISO, N.KDN_PREC_BF16
    a.B, a.T, a.H, a.K, a.V = 4, 4096, 18, 128, 128
    saved = lib.kdn_scan_saved_bytes(ctypes.byref(a))
    # status word + one chunk record per 64-chunk (128-byte swizzled bf16
    # tiles: T, scale*Q, scale*Q^T [64][64]; Qs, Kf, Wf [2][64][64];
    # three [128] fp32 gate factors in a 2 KiB slot) + the chunk-start states,
    # [128][64] bf16 per value tile of 64
    nt, bh = 4096 // 64, 72
    record = 3 * 64 * 128 + 3 * 64 * 256 + 2048
    state = 2 * 128 * 64 * 2
    assert saved == 256 + bh * nt * record + bh * nt * state
    ws = lib.kdn_scan_workspace_bytes(ctypes.byref(a))
    assert ws == 256 + bh * nt * state  # status word + chunk-end adjoints
    a.K = 64
    assert lib.kdn_scan_saved_bytes(ctypes.byref(a)) == 0


def test_invalid_arguments_are_rejected_without_launch(lib):
    a = N.KdnScanArgs()
    a.variant, a.precision = N.KDN_DIAG, N.KDN_PREC_BF16
    a.B, a.T, a.H, a.K, a.V = 1, 32, 1, 64, 64
    rc = lib.kdn_scan_fwd(ctypes.byref(a), None)
    assert rc == -1
    assert b"K and V must be 128" in lib.kdn_last_error()
    rc = lib.kdn_iso_gain_fwd(None, None, None, None, None, None, None, None, 1, 1, 1, 1.0, None, 0, None)
    assert rc == -1
    rc = lib.kdn_diag_gain_fwd(None, None, None, None, None, None, None, None, None, 1, 8, 1, 96, None, 0, None)
    assert rc == -1


def test_diag_gain_rejects_grids_beyond_the_launch_limit(lib):
    # B*H is a grid dimension of the diagonal gain kernels (limit 65535):
    # larger batches must fail validation, not the launch
    p = 16  # non-null placeholders: validation returns before touching memory
    rc = lib.kdn_diag_gain_fwd(p, p, p, p, p, None, p, p, None, 2, 64, 32768, 128, p, 1 << 40, None)
    assert rc == -1 and b"size too large" in lib.kdn_last_error()
    rc = lib.kdn_diag_gain_fwd_noalloc(p, p, p, p, p, p, p, None, 65536, 1, 1, 128, None)
    assert rc == -1 and b"size too large" in lib.kdn_last_error()
    rc = lib.kdn_diag_gain_bwd(p, p, p, p, p, None, p, p, p, p, None, p, p, p, p, None, None, 65536, 64, 1, 128,
                               p, 1 << 40, None)
    assert rc == -1 and b"size too large" in lib.kdn_last_error()


def test_diag_gain_sizes(lib):
    # segment carries (3 segments of 64 tokens) + the covariance before every token
    assert lib.kdn_diag_gain_carry_elems(2, 130, 3, 128) == 2 * 3 * 3 * 128 + 2 * 130 * 3 * 128
    assert lib.kdn_diag_gain_varlen_carry_elems(130, 3, 128, 4) == 3 * 4 * 128 + 130 * 3 * 128
    assert lib.kdn_diag_gain_workspace_bytes(2, 130, 3, 128) > 0


def test_operators_fail_loudly_without_cuda():
    import torch

    from kdn_b200.iso_kdn_chunk import _chunk_kda_precumsum_paired, iso_kdn_gain

    if torch.cuda.is_available():
        pytest.skip("checks the no-GPU behaviour")
    a = torch.rand(1, 4, 2)
    with pytest.raises(ValueError, match="CUDA"):
        iso_kdn_gain(a, a, a + 0.1, torch.ones(2), head_dim=128)
    q = torch.randn(1, 4, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA-only"):
        _chunk_kda_precumsum_paired(q, q, q, torch.zeros(1, 4, 2, 128), torch.rand(1, 4, 2))
