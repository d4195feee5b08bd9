"""Variable-length (packed) batches: sequences of different lengths packed
along T of a B = 1 batch, delimited by ``cu_seqlens`` (token offsets
[0, l0, l0 + l1, ..., total]), as in the flash-linear-attention varlen
convention the reference's dense path builds on.

Every sequence is an independent KDN stream: its memory state starts at
zero, its covariance at 1 / initial_precision, and its gate prefix
``g_cumsum`` restarts every chunk (64 tokens isotropic, 32 diagonal) counted
from the sequence's own first token.

The memory scans (``chunk_kalman_varlen``, ``chunk_kda_precumsum_varlen``)
and the diagonal gain (``diag_kdn_gain_varlen``) run natively: the kernels
walk a chunk table (``kdn_varlen_plan``, cached per offsets and device in a
``VarlenPlan``) in which every sequence owns its 64-token chunks, the last
one partial; the chunk-parallel kernels take one CTA per (chunk, head), the
sequential passes one CTA pair per (sequence, head), longest sequence first.
Each sequence gets exactly the arithmetic of a separate fixed-length call,
with no padding and no gathers.

The isotropic gain (``iso_kdn_gain_varlen``) runs the sequences as rows of
fixed-length batched calls (``map_sequences``): sequences are grouped by
length rounded up to ``bucket`` tokens (a multiple of 64); each group is
gathered into a ``[n_seq, L, ...]`` batch whose rows start at a sequence's
first token and are padded after its end with neutral tokens (unit
retention and observation noise, zero process noise), so that no padding
token changes a real token's output or gradient.  Outputs are gathered back
to the packed layout.  Its tensors are per-token scalars [1, T, H], so the
gathers are small.

``cu_seqlens`` may be a list, a CPU tensor or a CUDA tensor (read once on
the host: a CUDA tensor costs a device synchronisation).
"""
from __future__ import annotations

import collections
import ctypes

from typing import Callable, Sequence

import torch
from torch.autograd.function import once_differentiable

from . import _native as N
from . import diag_kdn_chunk, iso_kdn_chunk
from ._scan import ScanSaved, scan_backward, scan_forward

# gather plans by (offsets, bucket, device), least recently used last; bounded
# so that a stream of distinct packings cannot grow it without limit
_INDEX_CACHE: "collections.OrderedDict" = collections.OrderedDict()
_INDEX_CACHE_MAX = 64


def offsets(cu_seqlens) -> list[int]:
    """Host list of the token offsets; validates monotonicity."""
    cu = cu_seqlens.tolist() if isinstance(cu_seqlens, torch.Tensor) else list(cu_seqlens)
    cu = [int(x) for x in cu]
    if len(cu) < 2 or cu[0] != 0 or any(b <= a for a, b in zip(cu, cu[1:])):
        raise ValueError("cu_seqlens must start at 0 and increase strictly")
    return cu


def _plan(cu: list[int], bucket: int, chunk: int, device: torch.device):
    """Groups of sequences by padded length and the device index tensors that
    gather every group's padded rows in one pass (cached per offsets, bucket,
    gate chunk and device).  Returns ``(shapes, src, valid, src_g, hold, out)``:
    ``shapes`` lists ``(L, n_seq)`` per group; the gathered rows of all groups
    are concatenated, row i reading packed token ``src[i]`` (``valid[i]``) or
    padding; ``out[t]`` is the gathered row of packed token t."""
    key = (tuple(cu), bucket, chunk, str(device))
    plan = _INDEX_CACHE.get(key)
    if plan is not None:
        _INDEX_CACHE.move_to_end(key)
        return plan
    groups: dict[int, list[int]] = {}
    for i in range(len(cu) - 1):
        n = cu[i + 1] - cu[i]
        groups.setdefault(-(-n // bucket) * bucket, []).append(i)
    shapes, pos_l, start_l, len_l = [], [], [], []
    for L, seqs in sorted(groups.items()):
        shapes.append((L, len(seqs)))
        pos_l.append(torch.arange(L).repeat(len(seqs)))  # position inside the padded row
        start_l.append(torch.tensor([cu[i] for i in seqs]).repeat_interleave(L))
        len_l.append(torch.tensor([cu[i + 1] - cu[i] for i in seqs]).repeat_interleave(L))
    pos, start, length = torch.cat(pos_l), torch.cat(start_l), torch.cat(len_l)
    valid = pos < length
    src = torch.where(valid, start + pos, torch.zeros_like(pos))  # any in-range row where padded
    # gate prefix: the last real token's value up to the end of its chunk
    hold = pos < (length + chunk - 1) // chunk * chunk
    src_g = start + torch.minimum(pos, length - 1)
    out = torch.empty(cu[-1], dtype=torch.long)
    out[(start + pos)[valid]] = torch.nonzero(valid).squeeze(1)
    plan = (shapes, src.to(device), valid.to(device), src_g.to(device), hold.to(device), out.to(device))
    _INDEX_CACHE[key] = plan
    while len(_INDEX_CACHE) > _INDEX_CACHE_MAX:
        _INDEX_CACHE.popitem(last=False)
    return plan


class _Gather(torch.autograd.Function):
    """rows[i] = x[src[i]] where keep[i], else ``fill``.  Every token is the
    source of exactly one real row (``inv[t]``), so the gradient of x is a
    gather as well (held padding copies of a gate row carry no cotangent)."""

    @staticmethod
    def forward(ctx, x, src, keep, fill, inv):
        ctx.save_for_backward(inv)
        rows = x.index_select(0, src)
        mask = keep.view(-1, *([1] * (rows.dim() - 1)))
        return torch.where(mask, rows, torch.full((), fill, dtype=x.dtype, device=x.device))

    @staticmethod
    def backward(ctx, g):
        (inv,) = ctx.saved_tensors
        return g.index_select(0, inv), None, None, None, None


class _Scatter(torch.autograd.Function):
    """out[t] = rows[inv[t]]: the real rows back in packed order; the gradient
    of the rows is the gather of the packed gradient, zero on padding rows."""

    @staticmethod
    def forward(ctx, rows, inv, src, valid):
        ctx.save_for_backward(src, valid)
        return rows.index_select(0, inv)

    @staticmethod
    def backward(ctx, g):
        src, valid = ctx.saved_tensors
        d = g.index_select(0, src)
        mask = valid.view(-1, *([1] * (d.dim() - 1)))
        return torch.where(mask, d, torch.zeros((), dtype=d.dtype, device=d.device)), None, None, None


def map_sequences(fn: Callable, tensors: Sequence, cu_seqlens, *, pad: Sequence = (), bucket: int = 1024,
                  gate: int | None = None, chunk: int = 64):
    """Apply ``fn(*batched)`` to the sequences of packed ``[1, total, ...]``
    tensors (other arguments pass through unchanged) and return its output(s)
    in the packed layout.  ``pad[i]`` is the fill value of ``tensors[i]`` after
    a sequence's end (default 0); ``tensors[gate]``, a chunk-local gate prefix
    restarting every ``chunk`` tokens, is held at its last real value to the
    end of that chunk instead.  ``fn`` receives ``[n_seq, L, ...]`` batches and
    must return tensors of the same leading shape.  Each packed tensor is
    gathered once for all groups, and every gradient moves by a gather too
    (no scatter-add)."""
    if bucket <= 0 or bucket % 64:
        raise ValueError("bucket must be a positive multiple of 64")
    cu = offsets(cu_seqlens)
    packed = [t for t in tensors if isinstance(t, torch.Tensor) and t.dim() >= 2]
    if not packed:
        raise ValueError("no packed [1, T, ...] tensor")
    total = packed[0].shape[1]
    if cu[-1] != total or any(t.shape[0] != 1 or t.shape[1] != total for t in packed):
        raise ValueError(f"packed tensors must be [1, {cu[-1]}, ...] to match cu_seqlens")
    shapes, src, valid, src_g, hold, out_rows = _plan(cu, bucket, chunk, packed[0].device)
    sizes = [L * n for L, n in shapes]
    fills = list(pad) + [0.0] * (len(tensors) - len(pad))
    per_group = []  # per tensor: its [n, L, ...] batches, or the pass-through argument
    for i, (t, fill) in enumerate(zip(tensors, fills)):
        if isinstance(t, torch.Tensor) and t.dim() >= 2:
            rows = _Gather.apply(t[0], src_g if i == gate else src, hold if i == gate else valid, fill, out_rows)
            per_group.append([part.view(n, L, *t.shape[2:])
                              for part, (L, n) in zip(torch.split(rows, sizes), shapes)])
        else:
            per_group.append([t] * len(shapes))
    results, is_tuple = [], False
    for gi in range(len(shapes)):
        out = fn(*(arg[gi] for arg in per_group))
        is_tuple = isinstance(out, tuple)
        results.append(out if is_tuple else (out,))
    outs = []
    for j in range(len(results[0])):
        cat = torch.cat([res[j].reshape(-1, *res[j].shape[2:]) for res in results], 0)
        outs.append(_Scatter.apply(cat, out_rows, src, valid).unsqueeze(0))
    return tuple(outs) if is_tuple else outs[0]


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
        self.table = host.to(device)


def plan(cu_seqlens, device) -> VarlenPlan:
    """The (cached) plan of ``cu_seqlens`` on ``device``."""
    cu = offsets(cu_seqlens)
    key = (tuple(cu), str(torch.device(device)))
    p = _PLAN_CACHE.get(key)
    if p is None:
        p = VarlenPlan(cu, torch.device(device))
        _PLAN_CACHE[key] = p
        while len(_PLAN_CACHE) > _INDEX_CACHE_MAX:
            _PLAN_CACHE.popitem(last=False)
    else:
        _PLAN_CACHE.move_to_end(key)
    return p


def _check_packed(name: str, t: torch.Tensor, cu: tuple) -> None:
    if t.shape[0] != 1 or t.shape[1] != cu[-1]:
        raise ValueError(f"{name} must be a packed [1, {cu[-1]}, ...] batch to match cu_seqlens")


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
    vp = plan(cu_seqlens, q.device)
    _check_packed("q", q, vp.cu)
    return _IsoMemoryVarlenFunction.apply(q, k, v, g_cumsum, beta, scale, vp)


def iso_kdn_gain_varlen(a, omega, r, initial_precision, *, head_dim: int, cu_seqlens, out_dtype=None,
                        info_scale=None, bucket: int = 1024):
    """``iso_kdn_gain`` over a packed batch: the covariance restarts at every sequence."""
    def one(aa, w, rr):
        return iso_kdn_chunk.iso_kdn_gain(aa, w, rr, initial_precision, head_dim=head_dim, out_dtype=out_dtype,
                                          info_scale=info_scale)

    return map_sequences(one, (a, omega, r), cu_seqlens, pad=(1.0, 0.0, 1.0), bucket=bucket)


__all__ = ("chunk_kalman_varlen", "diag_kdn_gain_varlen", "chunk_kda_precumsum_varlen", "iso_kdn_gain_varlen",
           "VarlenPlan", "plan",
           "map_sequences", "offsets")
