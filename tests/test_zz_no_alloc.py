"""GPU test of kdn_diag_gain_fwd_noalloc, the entry point for callers that
cannot allocate device memory at call time (stream capture, allocation-free
plugin enqueue).  It must produce exactly what the workspace-taking
kdn_diag_gain_fwd produces, call after call, while keeping its scratch in the
library's static device array.  This file is collected last on purpose."""
import ctypes

import pytest
import torch

import oracle
from kdn_b200 import _native as N

pytestmark = pytest.mark.gpu


def _inputs(seed, B, T, H, K):
    d = oracle.make_diag_inputs(B, T, H, K=K, V=K, seed=seed)
    prec = 0.1 + torch.nn.functional.softplus(torch.randn(H, generator=torch.Generator().manual_seed(seed)))
    names = ("k_gain", "alpha", "omega", "r")
    return [d[n].cuda().contiguous() for n in names] + [prec.cuda()]


def _call(lib, fn, args, B, T, H, K, workspace):
    k, alpha, omega, r, prec = args
    kappa = torch.empty_like(k)
    carry = torch.empty(lib.kdn_diag_gain_carry_elems(B, T, H, K), device="cuda")
    p_final = torch.empty(B, H, K, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    outs = [t.data_ptr() for t in (kappa, carry, p_final)]
    ins = [t.data_ptr() for t in (k, alpha, omega, r, prec)]
    if workspace:
        ws = torch.empty(lib.kdn_diag_gain_workspace_bytes(B, T, H, K), dtype=torch.uint8, device="cuda")
        rc = fn(*ins, None, *outs, B, T, H, K, ws.data_ptr(), ws.numel(), stream)
    else:
        rc = fn(*ins, *outs, B, T, H, K, stream)
    assert rc == 0, lib.kdn_last_error()
    torch.cuda.synchronize()
    return kappa, carry, p_final


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    lib = N.load_library()
    # two calls in a row with different shapes and data share the static scratch
    for seed, (B, T, H, K) in ((3, (2, 300, 3, 128)), (4, (1, 1000, 2, 64))):
        args = _inputs(seed, B, T, H, K)
        ref = _call(lib, lib.kdn_diag_gain_fwd, args, B, T, H, K, workspace=True)
        got = _call(lib, lib.kdn_diag_gain_fwd_noalloc, args, B, T, H, K, workspace=False)
        for x, y in zip(got, ref):
            assert torch.allclose(x, y, rtol=1e-6, atol=0), (x - y).abs().max().item()


def test_noalloc_rejects_sizes_beyond_its_static_scratch():
    lib = N.load_library()
    x = torch.zeros(8, device="cuda")
    p = x.data_ptr()
    # 1 * 1 * ceil(600000 / 64) * 128 > 2^20 entries
    rc = lib.kdn_diag_gain_fwd_noalloc(p, p, p, p, p, p, p, None, 1, 600000, 1, 128, None)
    assert rc == -1
    assert b"exceeds the static scratch" in lib.kdn_last_error()
