"""Host side of the chunked memory scan: buffer allocation and the two calls
into ``kdn_scan_fwd`` / ``kdn_scan_bwd``.  Shared by the isotropic and the
diagonal operator modules and by the sequence-parallel driver."""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch

from . import _native as N

KD = 128


STATUS_GAVE_UP = 1  # a bounded wait ran out of polls: the call's results are invalid
STATUS_SLOW_WAIT = 2  # a wait needed more polls than KDN_B200_DEBUG_POLL_LIMIT (debug knob; results valid)


def status_word(buf: torch.Tensor) -> int:
    """The status word at the head of ``saved`` (forward) or the workspace
    (backward); reading it synchronises with the device."""
    return int(buf[:4].view(torch.int32).item())


def check_status(buf: torch.Tensor, what: str) -> None:
    """With ``KDN_B200_CHECK_STATUS=1``, synchronise and read the status word
    of the call: the kernels' bounded waits set ``STATUS_GAVE_UP`` when they
    gave up (the results of that call are then invalid) and
    ``STATUS_SLOW_WAIT`` when ``KDN_B200_DEBUG_POLL_LIMIT`` is set and a wait
    needed more polls than it.  Off by default (it costs a device round
    trip)."""
    if os.environ.get("KDN_B200_CHECK_STATUS", "0") != "1":
        return
    word = status_word(buf)
    if word & STATUS_GAVE_UP:
        raise RuntimeError(f"{what}: a bounded wait in the kernels gave up (status word {word}); results are invalid")
    if word:
        raise RuntimeError(f"{what}: a wait exceeded the debug poll limit KDN_B200_DEBUG_POLL_LIMIT "
                           f"(status word {word})")


@dataclass
class ScanSaved:
    """What the forward leaves for the backward (besides the inputs)."""

    saved: torch.Tensor  # uint8: T and Q per chunk (fp32), chunk-start states
    precision: int


def _args(variant, precision, q, v, scale, plan=None) -> N.KdnScanArgs:
    B, T, H, K = q.shape
    a = N.KdnScanArgs()
    a.variant = variant
    a.precision = precision
    a.B, a.T, a.H, a.K, a.V = B, T, H, K, v.shape[-1]
    a.scale = float(scale)
    if plan is not None:
        # packed variable-length batch: the plan's table on the device
        if precision != N.KDN_PREC_BF16:
            raise ValueError("packed variable-length batches run the bf16 precision only")
        a.varlen_table = plan.table.data_ptr()
        a.num_seqs = plan.num_seqs
        a.num_chunks = plan.num_chunks
    return a


def _streams(q, plan) -> int:
    """Leading size of the per-stream states: B, or the sequences of a packed batch."""
    return q.shape[0] if plan is None else plan.num_seqs


def scan_forward(variant, q, k, v, g, gate, scale, initial_state=None, want_final_state=False, plan=None):
    """Run the forward.  ``gate`` is beta [B,T,H] (iso) or kappa [B,T,H,K]
    (diag).  ``plan`` (a packed batch's ``kdn_b200.varlen.VarlenPlan``) makes
    the states per sequence.  Returns ``(o, final_state or None, ScanSaved)``."""
    N.require_cuda(q, k, v, g, gate)
    lib = N.load_library()
    prec = N.precision()
    a = _args(variant, prec, q, v, scale, plan)
    saved = N.byte_buffer(lib.kdn_scan_saved_bytes(ctypes.byref(a)), q.device)
    ws_bytes = lib.kdn_scan_workspace_bytes(ctypes.byref(a))
    if prec == N.KDN_PREC_FP32:
        ws = N.byte_buffer(ws_bytes, q.device)
    else:
        ws = None
    o = torch.empty(v.shape, dtype=torch.bfloat16 if variant == N.KDN_ISO else torch.float32, device=q.device)
    final = (torch.empty(_streams(q, plan), q.shape[2], KD, v.shape[-1], dtype=torch.float32, device=q.device)
             if want_final_state else None)
    a.q, a.k, a.v, a.g = q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr()
    if variant == N.KDN_ISO:
        a.beta = gate.data_ptr()
    else:
        a.kappa = gate.data_ptr()
    a.initial_state = N.ptr(initial_state)
    a.o = o.data_ptr()
    a.final_state = N.ptr(final)
    a.saved = saved.data_ptr()
    a.workspace = N.ptr(ws)
    a.workspace_bytes = ws.numel() if ws is not None else 0
    N.check(lib.kdn_scan_fwd(ctypes.byref(a), N.stream_of(q)), "kdn_scan_fwd")
    check_status(saved, "kdn_scan_fwd")
    return o, final, ScanSaved(saved, prec)


def scan_backward(variant, q, k, v, g, gate, scale, saved: ScanSaved, dO, d_final_state=None, want_d_initial=False,
                  plan=None):
    """Run the backward.  Returns ``(dq, dk, dv, dg, dgate, d_initial_state)``
    where dgate is dbeta (iso) or dkappa (diag)."""
    lib = N.load_library()
    a = _args(variant, saved.precision, q, v, scale, plan)
    ws = N.byte_buffer(lib.kdn_scan_workspace_bytes(ctypes.byref(a)), q.device)
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    dg = torch.empty_like(g)
    dgate = torch.empty_like(gate)
    dS0 = (
        torch.empty(_streams(q, plan), q.shape[2], KD, v.shape[-1], dtype=torch.float32, device=q.device)
        if want_d_initial
        else None
    )
    a.q, a.k, a.v, a.g = q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr()
    if variant == N.KDN_ISO:
        a.beta = gate.data_ptr()
        a.dbeta = dgate.data_ptr()
    else:
        a.kappa = gate.data_ptr()
        a.dkappa = dgate.data_ptr()
    a.saved = saved.saved.data_ptr()
    a.dO = dO.data_ptr()
    a.d_final_state = N.ptr(d_final_state)
    a.dq, a.dk, a.dv, a.dg = dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr()
    a.d_initial_state = N.ptr(dS0)
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel()
    N.check(lib.kdn_scan_bwd(ctypes.byref(a), N.stream_of(q)), "kdn_scan_bwd")
    check_status(ws, "kdn_scan_bwd")
    return dq, dk, dv, dg, dgate, dS0
