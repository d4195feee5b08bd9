"""The scan kernels' status word, exercised on the GPU without a fault.

Every mbarrier wait in the scan kernels polls a bounded number of times and
records a time-out in the call's status word, which the host reads.  A real
time-out cannot be provoked safely (a kernel that stops waiting for its own
copies could leave them in flight), so the library has a debug poll limit,
``KDN_B200_DEBUG_POLL_LIMIT``: a wait that needs more polls than it sets the
slow-wait bit and then keeps waiting up to the hard limit.  These tests set
it to 1 and check that the bit reaches the status word, that the host check
raises, that the results are still exact, and that the next call with the
knob off is clean.
"""
import ctypes

import pytest
import torch

import oracle
from kdn_b200 import _native as N
from kdn_b200 import _scan
from kdn_b200.iso_kdn_chunk import _chunk_kda_precumsum_paired

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _scan_calls(d):
    """One kdn_scan_fwd + kdn_scan_bwd through the C ABI with caller-owned
    buffers; returns the two status words and every output."""
    lib = N.load_library()
    q, k, v, g, beta, dO = (d[n].to(DEV).contiguous() for n in ("q", "k", "v", "g_cumsum", "beta", "dO"))
    a = _scan._args(N.KDN_ISO, N.KDN_PREC_BF16, q, v, 128 ** -0.5)
    saved = N.byte_buffer(lib.kdn_scan_saved_bytes(ctypes.byref(a)), q.device)
    ws = N.byte_buffer(lib.kdn_scan_workspace_bytes(ctypes.byref(a)), q.device)
    o = torch.empty_like(v)
    dq, dk, dv, dg, dbeta = (torch.empty_like(t) for t in (q, k, v, g, beta))
    a.q, a.k, a.v, a.g, a.beta = q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr()
    a.o, a.saved, a.dO = o.data_ptr(), saved.data_ptr(), dO.data_ptr()
    a.dq, a.dk, a.dv, a.dg, a.dbeta = dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), dbeta.data_ptr()
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    stream = N.stream_of(q)
    N.check(lib.kdn_scan_fwd(ctypes.byref(a), stream), "kdn_scan_fwd")
    fwd_word = _scan.status_word(saved)
    N.check(lib.kdn_scan_bwd(ctypes.byref(a), stream), "kdn_scan_bwd")
    bwd_word = _scan.status_word(ws)
    return fwd_word, bwd_word, (o, dq, dk, dv, dg, dbeta)


def test_debug_poll_limit_sets_the_status_word_and_results_stay_exact(monkeypatch):
    d = oracle.make_iso_inputs(1, 1024, 2, seed=5)
    monkeypatch.delenv("KDN_B200_DEBUG_POLL_LIMIT", raising=False)
    w0f, w0b, clean = _scan_calls(d)
    assert (w0f, w0b) == (0, 0)

    monkeypatch.setenv("KDN_B200_DEBUG_POLL_LIMIT", "1")
    w1f, w1b, flagged = _scan_calls(d)
    # no wait gave up (bit 0), and at least one needed more than one poll (bit 1)
    assert not (w1f | w1b) & _scan.STATUS_GAVE_UP
    assert (w1f | w1b) == _scan.STATUS_SLOW_WAIT, (w1f, w1b)
    # the slow waits still completed: the results are the clean call's (to
    # the last bits of fp32 partial sums the chunk backward adds atomically)
    for x, y in zip(flagged, clean):
        assert same(x, y)

    monkeypatch.delenv("KDN_B200_DEBUG_POLL_LIMIT")
    w2f, w2b, again = _scan_calls(d)
    assert (w2f, w2b) == (0, 0)
    for x, y in zip(again, clean):
        assert same(x, y)


def same(x, y):
    x, y = x.double(), y.double()
    return ((x - y).abs().max() / y.abs().max().clamp_min(1e-30)).item() < 1e-5


def test_host_status_check_raises_through_the_public_operator(monkeypatch):
    d = oracle.make_iso_inputs(1, 1024, 2, seed=6)
    leaves = [d[n].to(DEV).requires_grad_(True) for n in ("q", "k", "v", "g_cumsum", "beta")]
    monkeypatch.setenv("KDN_B200_CHECK_STATUS", "1")
    monkeypatch.setenv("KDN_B200_DEBUG_POLL_LIMIT", "1")
    with pytest.raises(RuntimeError, match="debug poll limit"):
        o = _chunk_kda_precumsum_paired(*leaves)
        o.backward(d["dO"].to(DEV))
    torch.cuda.synchronize()
    monkeypatch.delenv("KDN_B200_DEBUG_POLL_LIMIT")
    for t in leaves:
        t.grad = None
    o = _chunk_kda_precumsum_paired(*leaves)
    o.backward(d["dO"].to(DEV))
    torch.cuda.synchronize()
    assert all(t.grad is not None for t in leaves)
