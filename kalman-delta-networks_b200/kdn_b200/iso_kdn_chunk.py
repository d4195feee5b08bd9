"""Isotropic KDN operators on B200: drop-in replacements for

* ``iso_kdn_gain``                (lit_gpt/kdn_ops/iso_kdn_chunk.py:1966)
* ``_chunk_kda_precumsum_paired`` (lit_gpt/kdn_ops/iso_kdn_chunk.py:2242)

with the reference's signatures, validation messages, tensor layouts and
autograd contract.  Both run on the sm_100a kernels of ``libkdn_b200.so``;
there is no CPU or Triton path.
"""
from __future__ import annotations

import math
from numbers import Real

import torch

from . import _native as N
from ._scan import scan_backward, scan_forward


def _require_same_cuda_device(a: torch.Tensor, *named_tensors: tuple[str, torch.Tensor]) -> torch.device:
    if not a.is_cuda:
        raise ValueError(f"a must be a CUDA tensor; got device={a.device}")
    device = a.device
    for name, tensor in named_tensors:
        if not tensor.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor; got device={tensor.device}")
        if tensor.device != device:
            raise ValueError(
                f"all tensors must share a CUDA device; a is on {device}, but {name} is on {tensor.device}"
            )
    return device


def _iso_gain_forward(a, omega, r, initial_precision, *, out_dtype, save_state, posterior_scale,
                      initial_cov=None, want_final=False):
    """Forward scalar covariance scan; optional carried-in covariance [B,H] and
    final covariance out (sequence parallelism)."""
    B, T, H = a.shape
    N.require_cuda(a)
    lib = N.load_library()
    a32, w32, r32, p32 = (x.float().contiguous() for x in (a, omega, r, initial_precision))
    c32 = None if initial_cov is None else initial_cov.float().contiguous()
    gain = torch.empty((B, T, H), dtype=torch.float32, device=a.device)
    p_prev = torch.empty((B, T, H), dtype=torch.float32, device=a.device) if save_state else None
    p_final = torch.empty((B, H), dtype=torch.float32, device=a.device) if want_final else None
    ws = N.byte_buffer(lib.kdn_iso_gain_workspace_bytes(B, T, H), a.device)
    N.check(
        lib.kdn_iso_gain_fwd(
            a32.data_ptr(), w32.data_ptr(), r32.data_ptr(), p32.data_ptr(), N.ptr(c32), gain.data_ptr(),
            N.ptr(p_prev), N.ptr(p_final), B, T, H, float(posterior_scale), ws.data_ptr(), ws.numel(),
            N.stream_of(a),
        ),
        "kdn_iso_gain_fwd",
    )
    return gain.to(out_dtype), p_prev, p_final


def _iso_gain_backward(a, omega, r, initial_precision, dgain, p_prev, *, posterior_scale, initial_cov=None,
                       d_final_cov=None, want_d_initial=False):
    B, T, H = a.shape
    lib = N.load_library()
    a32, w32, r32, p32, d32 = (x.float().contiguous() for x in (a, omega, r, initial_precision, dgain))
    dfc = None if d_final_cov is None else d_final_cov.float().contiguous()
    da = torch.empty((B, T, H), dtype=torch.float32, device=a.device)
    domega = torch.empty_like(da)
    dr = torch.empty_like(da)
    dinit = torch.empty((H,), dtype=torch.float32, device=a.device)
    dic = torch.empty((B, H), dtype=torch.float32, device=a.device) if want_d_initial else None
    ws = N.byte_buffer(lib.kdn_iso_gain_workspace_bytes(B, T, H), a.device)
    N.check(
        lib.kdn_iso_gain_bwd(
            a32.data_ptr(), w32.data_ptr(), r32.data_ptr(), p32.data_ptr(), N.ptr(initial_cov), d32.data_ptr(),
            p_prev.data_ptr(), N.ptr(dfc), da.data_ptr(), domega.data_ptr(), dr.data_ptr(), dinit.data_ptr(),
            N.ptr(dic), B, T, H, float(posterior_scale), ws.data_ptr(), ws.numel(), N.stream_of(a),
        ),
        "kdn_iso_gain_bwd",
    )
    return da.to(a.dtype), domega.to(omega.dtype), dr.to(r.dtype), dinit.to(initial_precision.dtype), dic


class _IsoKDNGainFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, omega, r, initial_precision, out_dtype, posterior_scale, needs_backward):
        gain, p_prev, _ = _iso_gain_forward(
            a, omega, r, initial_precision, out_dtype=out_dtype, save_state=needs_backward,
            posterior_scale=posterior_scale,
        )
        ctx.posterior_scale = posterior_scale
        ctx.has_saved_state = needs_backward
        if needs_backward:
            ctx.save_for_backward(a, omega, r, initial_precision, p_prev)
        return gain

    @staticmethod
    def backward(ctx, dgain):
        if dgain is None:
            return None, None, None, None, None, None, None
        if not ctx.has_saved_state:
            raise RuntimeError("Isotropic KDN gain backward called after a no-save forward")
        a, omega, r, initial_precision, p_prev = ctx.saved_tensors
        da, domega, dr, dinit, _ = _iso_gain_backward(
            a, omega, r, initial_precision, dgain, p_prev, posterior_scale=ctx.posterior_scale
        )
        needs = ctx.needs_input_grad
        return (
            da if needs[0] else None,
            domega if needs[1] else None,
            dr if needs[2] else None,
            dinit if needs[3] else None,
            None,
            None,
            None,
        )


@torch.compiler.disable
def iso_kdn_gain(
    a: torch.Tensor,
    omega: torch.Tensor,
    r: torch.Tensor,
    initial_precision: torch.Tensor,
    *,
    head_dim: int,
    out_dtype: torch.dtype | None = None,
    info_scale: Real | None = None,
) -> torch.Tensor:
    """Differentiable Isotropic KDN scalar write gate (see iso_kdn_chunk.py:1976-1990).

    a, omega, r: [B, T, H]; initial_precision: [H].  The scalar covariance
    scan runs in fp32 on the GPU; ``posterior_scale = info_scale / head_dim``.
    """
    if a.ndim != 3:
        raise ValueError(f"a must have shape [B,T,H], got {tuple(a.shape)}")
    if omega.shape != a.shape or r.shape != a.shape:
        raise ValueError(
            f"a, omega, and r must share shape [B,T,H]; got "
            f"a={tuple(a.shape)}, omega={tuple(omega.shape)}, r={tuple(r.shape)}"
        )
    H = a.shape[-1]
    if initial_precision.ndim != 1 or initial_precision.shape[0] != H:
        raise ValueError(f"initial_precision must have shape [{H}], got {tuple(initial_precision.shape)}")
    _require_same_cuda_device(a, ("omega", omega), ("r", r), ("initial_precision", initial_precision))
    if isinstance(head_dim, bool) or not isinstance(head_dim, int):
        raise TypeError(f"head_dim must be a positive int, got {type(head_dim).__name__}")
    if head_dim <= 0:
        raise ValueError(f"head_dim must be positive, got {head_dim}")
    if out_dtype is None:
        out_dtype = torch.float32
    if info_scale is None:
        resolved_info_scale = float(head_dim)
    else:
        if isinstance(info_scale, bool) or not isinstance(info_scale, Real):
            raise TypeError(f"info_scale must be a positive finite real, got {type(info_scale).__name__}")
        resolved_info_scale = float(info_scale)
        if not math.isfinite(resolved_info_scale) or resolved_info_scale <= 0:
            raise ValueError(f"info_scale must be positive and finite, got {info_scale!r}")
    posterior_scale = resolved_info_scale / float(head_dim)
    needs_backward = torch.is_grad_enabled() and any(
        t.requires_grad for t in (a, omega, r, initial_precision)
    )
    return _IsoKDNGainFunction.apply(
        a.contiguous(), omega.contiguous(), r.contiguous(), initial_precision.contiguous(),
        out_dtype, posterior_scale, needs_backward,
    )


class _ChunkKDAPrecumsumFunction(torch.autograd.Function):
    """Isotropic memory scan: q, k L2-normalised in the kernel, kappa = beta k_hat.

    Saves the raw inputs plus the kernel's per-chunk state (chunk-start
    memories, triangular solve T and scores Q) for the backward, which
    returns ``(dq, dk, dv, dg_pre_reverse, dbeta, None)`` with ``dg`` in
    natural-log coordinates before the reverse chunk cumsum
    (iso_kdn_chunk.py:2180-2186)."""

    @staticmethod
    def forward(ctx, q, k, v, g_cumsum, beta, scale):
        in_dtype = q.dtype
        qb, kb, vb = (x.to(torch.bfloat16).contiguous() for x in (q, k, v))
        g = g_cumsum.contiguous()
        b = beta.float().contiguous()
        o, _, saved = scan_forward(N.KDN_ISO, qb, kb, vb, g, b, scale)
        ctx.save_for_backward(qb, kb, vb, g, b, saved.saved)
        ctx.precision = saved.precision
        ctx.scale = scale
        ctx.dtypes = (in_dtype, k.dtype, v.dtype, beta.dtype)
        return o.to(in_dtype)

    @staticmethod
    def backward(ctx, do):
        from ._scan import ScanSaved

        qb, kb, vb, g, b, saved = ctx.saved_tensors
        dO = do.to(torch.bfloat16).contiguous()
        dq, dk, dv, dg, dbeta, _ = scan_backward(
            N.KDN_ISO, qb, kb, vb, g, b, ctx.scale, ScanSaved(saved, ctx.precision), dO
        )
        qd, kd, vd, bd = ctx.dtypes
        return dq.to(qd), dk.to(kd), dv.to(vd), dg.to(g.dtype), dbeta.to(bd), None


@torch.compiler.disable
def _chunk_kda_precumsum_paired(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g_cumsum: torch.Tensor,
    beta: torch.Tensor,
    scale: float | None = None,
) -> torch.Tensor:
    """Isotropic KDN memory scan on the fixed-length path (see iso_kdn_chunk.py:2250-2256).

    ``g_cumsum`` is the 64-local base-2 prefix of ln(alpha); the backward
    returns the natural-log cotangent its producer expects.  The kernels take
    bf16 q/k/v (other floating dtypes are rounded to bf16) with
    K = V = 128.
    """
    if q.ndim != 4 or q.shape != k.shape:
        raise ValueError(f"q and k must share [B,T,H,K], got {tuple(q.shape)} and {tuple(k.shape)}")
    B, T, H, K = q.shape
    if min(B, T, H, K) == 0:
        raise ValueError("_chunk_kda_precumsum_paired requires non-empty B,T,H,K dimensions")
    if v.ndim != 4 or v.shape[:3] != (B, T, H):
        raise NotImplementedError("_chunk_kda_precumsum_paired does not support GVA; v must have q's B,T,H")
    if v.shape[-1] == 0:
        raise ValueError("_chunk_kda_precumsum_paired requires a non-empty value dimension")
    if g_cumsum.shape != (B, T, H, K):
        raise ValueError(f"g_cumsum must have shape {(B, T, H, K)}, got {tuple(g_cumsum.shape)}")
    if beta.shape != (B, T, H):
        raise ValueError(f"beta must have shape {(B, T, H)}, got {tuple(beta.shape)}")
    if K > 256:
        raise ValueError(f"KDA supports key head dimension <=256, got {K}")
    if g_cumsum.dtype != torch.float32:
        raise TypeError(f"g_cumsum must be FP32 base-2 cumulative gate, got {g_cumsum.dtype}")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError(f"q, k, and v must share a dtype, got {q.dtype}, {k.dtype}, {v.dtype}")
    tensors = (q, k, v, g_cumsum, beta)
    if not all(x.is_cuda for x in tensors):
        raise ValueError("_chunk_kda_precumsum_paired is CUDA-only")
    if len({x.device for x in tensors}) != 1:
        raise ValueError("all _chunk_kda_precumsum_paired tensors must be on the same CUDA device")
    if K != 128 or v.shape[-1] != 128:
        raise ValueError(f"kdn_b200 kernels support K = V = 128, got K={K}, V={v.shape[-1]}")
    if scale is None:
        scale = K ** -0.5
    return _ChunkKDAPrecumsumFunction.apply(q, k, v, g_cumsum, beta, scale)


__all__ = ("_chunk_kda_precumsum_paired", "iso_kdn_gain")
