"""Variable-length (packed) batches: sequences of different lengths packed
along T of a B = 1 batch, delimited by ``cu_seqlens`` (token offsets
[0, l0, l0 + l1, ..., total]), as in the flash-linear-attention varlen
convention the reference's dense path builds on.

Every sequence is an independent KDN stream: its memory state starts at
zero, its covariance at 1 / initial_precision,
and its gate prefix ``g_cumsum`` restarts every chunk (64 tokens isotropic,
32 diagonal) counted from the sequence's own first token.  Each sequence
therefore runs as its own B = 1 call of the fixed-length operators, which
keeps the chunk boundaries and the mathematics identical; the calls are
spread over a pool of CUDA streams so that the sequential passes of
different sequences run at the same time.  Autograd runs each sequence's
backward on the stream of its forward.  Outputs are concatenated along T.

``cu_seqlens`` may be a list, a CPU tensor or a CUDA tensor (read once on
the host: a CUDA tensor costs a device synchronisation).
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch

from . import diag_kdn_chunk, iso_kdn_chunk

_POOL: dict[int, list[torch.cuda.Stream]] = {}


def _streams(device: torch.device, n: int) -> list[torch.cuda.Stream]:
    key = device.index if device.index is not None else torch.cuda.current_device()
    pool = _POOL.setdefault(key, [])
    while len(pool) < n:
        pool.append(torch.cuda.Stream(device))
    return pool[:n]


def join(device=None) -> None:
    """Make the current stream wait for every pool stream of ``device``: call
    after ``backward`` when the next work (or a CUDA graph capture) must see
    all per-sequence gradients on the current stream."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    key = device.index if device.index is not None else torch.cuda.current_device()
    cur = torch.cuda.current_stream(device)
    for s in _POOL.get(key, []):
        cur.wait_stream(s)


def offsets(cu_seqlens) -> list[int]:
    """Host list of the token offsets; validates monotonicity."""
    cu = cu_seqlens.tolist() if isinstance(cu_seqlens, torch.Tensor) else list(cu_seqlens)
    cu = [int(x) for x in cu]
    if len(cu) < 2 or cu[0] != 0 or any(b <= a for a, b in zip(cu, cu[1:])):
        raise ValueError("cu_seqlens must start at 0 and increase strictly")
    return cu


def map_sequences(fn: Callable, tensors: Sequence, cu_seqlens, *, streams: int = 4):
    """Apply ``fn(*slices)`` to every sequence (slices along dim 1 of the
    [1, T, ...] tensors; other arguments pass through) on a pool of streams and
    concatenate each output along dim 1."""
    cu = offsets(cu_seqlens)
    packed = [t for t in tensors if isinstance(t, torch.Tensor) and t.dim() >= 2]
    if not packed:
        raise ValueError("no packed [1, T, ...] tensor")
    total = packed[0].shape[1]
    if cu[-1] != total or any(t.shape[0] != 1 or t.shape[1] != total for t in packed):
        raise ValueError(f"packed tensors must be [1, {cu[-1]}, ...] to match cu_seqlens")
    device = packed[0].device
    main = torch.cuda.current_stream(device)
    pool = _streams(device, min(streams, len(cu) - 1))
    for s in pool:
        s.wait_stream(main)
    outs = []
    for i in range(len(cu) - 1):
        s = pool[i % len(pool)]
        with torch.cuda.stream(s):
            args = [t[:, cu[i]:cu[i + 1]] if isinstance(t, torch.Tensor) and t.dim() >= 2 else t for t in tensors]
            outs.append(fn(*args))
    for s in pool:
        main.wait_stream(s)
    for o in outs:  # made on side streams, read by the concatenation on the main one
        for t in (o if isinstance(o, tuple) else (o,)):
            t.record_stream(main)
    if isinstance(outs[0], tuple):
        return tuple(torch.cat([o[j] for o in outs], dim=1) for j in range(len(outs[0])))
    return torch.cat(outs, dim=1)


def chunk_kalman_varlen(q_memory, k_memory, kappa, v, g_cumsum, scale: float, cu_seqlens, *, streams: int = 4):
    """``chunk_kalman`` over a packed batch (fp32 output [1, T, H, V])."""
    def one(q, k, kap, vv, g):
        return diag_kdn_chunk.chunk_kalman(q.contiguous(), k.contiguous(), kap.contiguous(), vv.contiguous(),
                                           g.contiguous(), scale)

    return map_sequences(one, (q_memory, k_memory, kappa, v, g_cumsum), cu_seqlens, streams=streams)


def diag_kdn_gain_varlen(k_gain, alpha, omega, r, initial_precision, omega_raw, r_raw, cu_seqlens, *,
                         streams: int = 4):
    """``_diag_kdn_gain`` over a packed batch: the covariance restarts at every sequence."""
    def one(kg, a, w, rr, wr, rrr):
        return diag_kdn_chunk._diag_kdn_gain(kg.contiguous(), a.contiguous(), w.contiguous(), rr.contiguous(),
                                            initial_precision, wr.contiguous(), rrr.contiguous())

    return map_sequences(one, (k_gain, alpha, omega, r, omega_raw, r_raw), cu_seqlens, streams=streams)


def chunk_kda_precumsum_varlen(q, k, v, g_cumsum, beta, scale: float | None = None, *, cu_seqlens,
                               streams: int = 4):
    """``_chunk_kda_precumsum_paired`` over a packed batch."""
    def one(qq, kk, vv, g, b):
        return iso_kdn_chunk._chunk_kda_precumsum_paired(qq.contiguous(), kk.contiguous(), vv.contiguous(),
                                                         g.contiguous(), b.contiguous(), scale)

    return map_sequences(one, (q, k, v, g_cumsum, beta), cu_seqlens, streams=streams)


def iso_kdn_gain_varlen(a, omega, r, initial_precision, *, head_dim: int, cu_seqlens, out_dtype=None,
                        info_scale=None, streams: int = 4):
    """``iso_kdn_gain`` over a packed batch: the covariance restarts at every sequence."""
    def one(aa, w, rr):
        return iso_kdn_chunk.iso_kdn_gain(aa.contiguous(), w.contiguous(), rr.contiguous(), initial_precision,
                                          head_dim=head_dim, out_dtype=out_dtype, info_scale=info_scale)

    return map_sequences(one, (a, omega, r), cu_seqlens, streams=streams)


__all__ = ("chunk_kalman_varlen", "diag_kdn_gain_varlen", "chunk_kda_precumsum_varlen", "iso_kdn_gain_varlen",
           "map_sequences", "offsets", "join")
