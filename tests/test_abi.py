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


def test_varlen_scan_sizes_and_validation(lib):
    """A packed batch sizes its saved state by global chunks; the C ABI
    rejects a packed batch with B > 1, the fp32 precision, a missing table or
    a partial-pass mode before launching anything."""
    cu = (ctypes.c_int64 * 4)(0, 70, 75, 203)  # chunks: 2 + 1 + 2
    nc = ctypes.c_int64(0)
    assert lib.kdn_varlen_plan(ctypes.cast(cu, ctypes.c_void_p), 3, None, 0, ctypes.byref(nc)) == 0
    assert nc.value == 5
    table = (ctypes.c_int32 * lib.kdn_varlen_table_len(3, 5))()
    assert lib.kdn_varlen_plan(ctypes.cast(cu, ctypes.c_void_p), 3, ctypes.cast(table, ctypes.c_void_p),
                               len(table), ctypes.byref(nc)) == 0
    assert list(table) == [0, 70, 75, 203, 0, 2, 3, 5, 2, 0, 1, 0, 0, 1, 2, 2]

    def args(**kw):
        a = N.KdnScanArgs()
        a.variant, a.precision = N.KDN_DIAG, N.KDN_PREC_BF16
        a.B, a.T, a.H, a.K, a.V = 1, 203, 2, 128, 128
        a.varlen_table, a.num_seqs, a.num_chunks = ctypes.addressof(table), 3, 5
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    fixed = N.KdnScanArgs()
    fixed.variant, fixed.precision = N.KDN_DIAG, N.KDN_PREC_BF16
    fixed.B, fixed.T, fixed.H, fixed.K, fixed.V = 1, 5 * 64, 2, 128, 128
    # five global chunks hold what a 320-token fixed batch's five chunks hold
    # (records and states), the gate prefix copy is per token
    packed = lib.kdn_scan_saved_bytes(ctypes.byref(args()))
    assert packed > 0 and packed < lib.kdn_scan_saved_bytes(ctypes.byref(fixed))
    for bad in (dict(B=2), dict(precision=N.KDN_PREC_FP32), dict(varlen_table=None), dict(num_chunks=2)):
        assert lib.kdn_scan_saved_bytes(ctypes.byref(args(**bad))) == 0, bad
        assert lib.kdn_scan_fwd(ctypes.byref(args(**bad)), None) == -1, bad
        assert b"packed batch" in lib.kdn_last_error()
    a = args(mode=N.KDN_SCAN_FWD_RECORDS, q=1, k=1, v=1, g=1, kappa=1, saved=1)
    assert lib.kdn_scan_fwd(ctypes.byref(a), None) == -1
    assert b"mode 0 only" in lib.kdn_last_error()


def test_varlen_gain_validation(lib):
    p = ctypes.c_void_p(16)
    assert lib.kdn_diag_gain_fwd_varlen(p, p, p, p, p, None, p, p, None, 100, 2, 128, None, 2, 3, p, 1 << 30,
                                        None) == -1
    assert b"kdn_varlen_plan table" in lib.kdn_last_error()
    assert lib.kdn_iso_gain_fwd_varlen(p, p, p, p, None, p, p, None, 100, 2, 1.0, p, 2, 101, p, 1 << 30,
                                       None) == -1  # longest sequence longer than T
    assert lib.kdn_iso_gain_varlen_workspace_bytes(3, 130, 2) == lib.kdn_iso_gain_workspace_bytes(3, 130, 2)
