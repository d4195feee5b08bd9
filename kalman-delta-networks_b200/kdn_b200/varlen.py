"""Variable-length (packed) batches: sequences of different lengths packed
along T of a B = 1 batch, delimited by ``cu_seqlens`` (token offsets
[0, l0, l0 + l1, ..., total]), as in the flash-linear-attention varlen
convention the reference's dense path builds on.

Every sequence is an independent KDN stream: its memory state starts at
zero, its covariance at 1 / initial_precision, and its gate prefix
``g_cumsum`` restarts every chunk (64 tokens isotropic, 32 diagonal) counted
from the sequence's own first token.

The memory scans (``chunk_kalman_varlen``, ``chunk_kda_precumsum_varlen``)
and the gains (``diag_kdn_gain_varlen``, ``iso_kdn_gain_varlen``) run
natively: the kernels walk a table (``kdn_varlen_plan``, cached per offsets
and device in a ``VarlenPlan``) in which every sequence owns its 64-token
chunks, the last one partial; the chunk-parallel kernels take one CTA per
(chunk, head), the sequential passes one CTA pair per (sequence, head),
longest sequence first, and the isotropic gain one stream per sequence.
Each sequence gets exactly the arithmetic of a separate fixed-length call,
with no padding and no gathers.

``cu_seqlens`` may be a list, a CPU tensor or a CUDA tensor (read once on
the host: a CUDA tensor costs a device synchronisation).
"""
from __future__ import annotations

import collections
import ctypes

import torch
from torch.autograd.function import once_differentiable

from . import _native as N
from . import diag_kdn_chunk, iso_kdn_chunk
from ._scan import ScanSaved, scan_backward, scan_forward

_PLAN_CACHE_MAX = 64  # plans cached per (offsets, device), least recently used first out


def offsets(cu_seqlens) -> list[int]:
    """Host list of the token offsets; validates monotonicity."""
    cu = cu_seqlens.tolist() if isinstance(cu_seqlens, torch.Tensor) else list(cu_seqlens)
    cu = [int(x) for x in cu]
    if len(cu) < 2 or cu[0] != 0 or any(b <= a for a, b in zip(cu, cu[1:])):
        raise ValueError("cu_seqlens must start at 0 and increase strictly")
    return cu


# --------------------------------------------------------------------------
# Native packed batches: the chunk table and the operators that walk it

_PLAN_CACHE: "collections.OrderedDict" = collections.OrderedDict()


class VarlenPlan:
    """The ``kdn_varlen_plan`` table of one packing on one device: token
    offsets, each sequence's first global 64-token chunk, the sequences by
    decreasing length and each chunk's sequence (int32, on the device)."""

    def __init__(self, cu: list[int], device: torch.device):
        lib = N.load_library()
        n = len(cu) - 1
        cu_host = (ctypes.c_int64 * len(cu))(*cu)
        nc = ctypes.c_int64(0)
        N.check(lib.kdn_varlen_plan(ctypes.cast(cu_host, ctypes.c_void_p), n, None, 0, ctypes.byref(nc)),
                "kdn_varlen_plan")
        length = lib.kdn_varlen_table_len(n, nc.value)
        host = torch.empty(length, dtype=torch.int32)
        N.check(lib.kdn_varlen_plan(ctypes.cast(cu_host, ctypes.c_void_p), n, host.data_ptr(), length,
                                    ctypes.byref(nc)), "kdn_varlen_plan")
        self.cu = tuple(cu)
        self.num_seqs = n
        self.num_chunks = int(nc.value)
        self.max_len = max(b - a for a, b in zip(cu, cu[1:]))
        self.table = host.to(device)


def plan(cu_seqlens, device) -> VarlenPlan:
    """The (cached) plan of ``cu_seqlens`` on ``device``."""
    cu = offsets(cu_seqlens)
    key = (tuple(cu), str(torch.device(device)))
    p = _PLAN_CACHE.get(key)
    if p is None:
        p = VarlenPlan(cu, torch.device(device))
        _PLAN_CACHE[key] = p
        while len(_PLAN_CACHE) > _PLAN_CACHE_MAX:
            _PLAN_CACHE.popitem(last=False)
    else:
        _PLAN_CACHE.move_to_end(key)
    return p


def _check_packed(name: str, t: torch.Tensor, cu: tuple) -> None:
    if t.shape[0] != 1 or t.shape[1] != cu[-1]:
        raise ValueError(f"{name} must be a packed [1, {cu[-1]}, ...] batch to match cu_seqlens")


def _check_width(*tensors: torch.Tensor) -> None:
    if any(t.shape[-1] != 128 for t in tensors):
        raise ValueError("packed batches run K = V = 128")


class _DiagGainVarlenFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, k, alpha, omega, r, initial_precision, omega_raw, r_raw, vp):
        kappa, carry, _ = diag_kdn_chunk._gain_forward(k, alpha, omega, r, initial_precision, plan=vp)
        ctx.save_for_backward(k, alpha, omega, r, initial_precision, omega_raw, r_raw, carry)
        ctx.vp = vp
        ctx.set_materialize_grads(False)
        return kappa

    @staticmethod
    @once_differentiable
    def backward(ctx, dkappa):
        k, alpha, omega, r, initial_precision, omega_raw, r_raw, carry = ctx.saved_tensors
        needs = ctx.needs_input_grad
        dk, dalpha, domega_raw, dr_raw, dinit, _ = diag_kdn_chunk._gain_backward(
            k, alpha, omega, r, initial_precision, omega_raw, r_raw, dkappa, carry, need_initial=needs[4],
            plan=ctx.vp)
        return (dk if needs[0] else None, dalpha if needs[1] else None, None, None, dinit if needs[4] else None,
                domega_raw if needs[5] else None, dr_raw if needs[6] else None, None)


def diag_kdn_gain_varlen(k_gain, alpha, omega, r, initial_precision, omega_raw, r_raw, cu_seqlens):
    """``_diag_kdn_gain`` over a packed batch: the covariance restarts at every
    sequence; ``initial_precision`` [H] is shared and collects every
    sequence's cotangent."""
    diag_kdn_chunk._validate_diag_kdn_gain_inputs(k_gain, alpha, omega, r, initial_precision, omega_raw, r_raw)
    vp = plan(cu_seqlens, k_gain.device)
    _check_packed("k_gain", k_gain, vp.cu)
    return _DiagGainVarlenFunction.apply(k_gain, alpha, omega.detach(), r.detach(), initial_precision, omega_raw,
                                         r_raw, vp)


class _DiagMemoryVarlenFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, kappa, v, g_cumsum, scale, vp):
        o, _, saved = scan_forward(N.KDN_DIAG, q, k, v, g_cumsum, kappa, scale, plan=vp)
        ctx.save_for_backward(q, k, kappa, v, g_cumsum, saved.saved)
        ctx.precision, ctx.scale, ctx.vp = saved.precision, scale, vp
        ctx.set_materialize_grads(False)
        return o

    @staticmethod
    @once_differentiable
    def backward(ctx, do):
        q, k, kappa, v, g_cumsum, saved = ctx.saved_tensors
        if do is None:
            return None, None, None, None, None, None, None
        do = do.contiguous()
        if do.shape != q.shape or do.dtype != torch.float32:
            raise TypeError("DiagKDN output cotangent must be FP32 BTHK")
        dq, dk, dv, dG, dkappa, _ = scan_backward(N.KDN_DIAG, q, k, v, g_cumsum, kappa, ctx.scale,
                                                  ScanSaved(saved, ctx.precision), do, plan=ctx.vp)
        return dq, dk, dkappa, dv, dG, None, None


def chunk_kalman_varlen(q_memory, k_memory, kappa, v, g_cumsum, scale: float, cu_seqlens):
    """``chunk_kalman`` over a packed batch (fp32 output [1, T, H, V]); the
    gate prefix restarts every 32 tokens from each sequence's first token."""
    diag_kdn_chunk._validate_diag_kdn_memory_inputs(q_memory, k_memory, kappa, v, g_cumsum, scale)
    _check_width(q_memory, v)
    vp = plan(cu_seqlens, q_memory.device)
    _check_packed("q_memory", q_memory, vp.cu)
    return _DiagMemoryVarlenFunction.apply(q_memory, k_memory, kappa, v, g_cumsum, scale, vp)


class _IsoMemoryVarlenFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g_cumsum, beta, scale, vp):
        dtypes = (q.dtype, k.dtype, v.dtype, beta.dtype)
        qb, kb, vb = (x.to(torch.bfloat16).contiguous() for x in (q, k, v))
        g, b = g_cumsum.contiguous(), beta.float().contiguous()
        o, _, saved = scan_forward(N.KDN_ISO, qb, kb, vb, g, b, scale, plan=vp)
        ctx.save_for_backward(qb, kb, vb, g, b, saved.saved)
        ctx.precision, ctx.scale, ctx.vp, ctx.dtypes = saved.precision, scale, vp, dtypes
        return o.to(dtypes[0])

    @staticmethod
    def backward(ctx, do):
        qb, kb, vb, g, b, saved = ctx.saved_tensors
        dq, dk, dv, dg, dbeta, _ = scan_backward(N.KDN_ISO, qb, kb, vb, g, b, ctx.scale,
                                                 ScanSaved(saved, ctx.precision),
                                                 do.to(torch.bfloat16).contiguous(), plan=ctx.vp)
        qd, kd, vd, bd = ctx.dtypes
        return dq.to(qd), dk.to(kd), dv.to(vd), dg.to(g.dtype), dbeta.to(bd), None, None


def chunk_kda_precumsum_varlen(q, k, v, g_cumsum, beta, scale: float | None = None, *, cu_seqlens):
    """``_chunk_kda_precumsum_paired`` over a packed batch; the 64-local gate
    prefix restarts at every sequence's first token."""
    scale = iso_kdn_chunk._validate_chunk_kda_inputs(q, k, v, g_cumsum, beta, scale)
    _check_width(q, v)
    vp = plan(cu_seqlens, q.device)
    _check_packed("q", q, vp.cu)
    return _IsoMemoryVarlenFunction.apply(q, k, v, g_cumsum, beta, scale, vp)


class _IsoGainVarlenFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, omega, r, initial_precision, out_dtype, posterior_scale, vp):
        gain, p_prev, _ = iso_kdn_chunk._iso_gain_forward(a, omega, r, initial_precision, out_dtype=out_dtype,
                                                          save_state=True, posterior_scale=posterior_scale, plan=vp)
        ctx.save_for_backward(a, omega, r, initial_precision, p_prev)
        ctx.posterior_scale, ctx.vp = posterior_scale, vp
        return gain

    @staticmethod
    def backward(ctx, dgain):
        if dgain is None:
            return None, None, None, None, None, None, None
        a, omega, r, initial_precision, p_prev = ctx.saved_tensors
        da, domega, dr, dinit, _ = iso_kdn_chunk._iso_gain_backward(
            a, omega, r, initial_precision, dgain, p_prev, posterior_scale=ctx.posterior_scale, plan=ctx.vp)
        return da, domega, dr, dinit, None, None, None


def iso_kdn_gain_varlen(a, omega, r, initial_precision, *, head_dim: int, cu_seqlens, out_dtype=None,
                        info_scale=None):
    """``iso_kdn_gain`` over a packed batch: the covariance restarts at every
    sequence; ``initial_precision`` [H] is shared and collects every
    sequence's cotangent."""
    out_dtype, posterior_scale = iso_kdn_chunk._validate_iso_gain_inputs(a, omega, r, initial_precision, head_dim,
                                                                         out_dtype, info_scale)
    vp = plan(cu_seqlens, a.device)
    _check_packed("a", a, vp.cu)
    return _IsoGainVarlenFunction.apply(a.contiguous(), omega.contiguous(), r.contiguous(),
                                        initial_precision.contiguous(), out_dtype, posterior_scale, vp)


__all__ = ("chunk_kalman_varlen", "diag_kdn_gain_varlen", "chunk_kda_precumsum_varlen", "iso_kdn_gain_varlen",
           "VarlenPlan", "plan", "offsets")
