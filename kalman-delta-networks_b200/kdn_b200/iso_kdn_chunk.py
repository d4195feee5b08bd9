"""Isotropic KDN operators on B200: drop-in replacements for

* ``_iso_kdn_gate_precumsum_paired`` (lit_gpt/kdn_ops/iso_kdn_chunk.py:1396)
* ``iso_kdn_gain``                   (lit_gpt/kdn_ops/iso_kdn_chunk.py:1966)
* ``_chunk_kda_precumsum_paired``    (lit_gpt/kdn_ops/iso_kdn_chunk.py:2242)

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
                      initial_cov=None, want_final=False, plan=None):
    """Forward scalar covariance scan; optional carried-in covariance [B,H] and
    final covariance out (sequence parallelism).  ``plan`` (a packed batch's
    ``kdn_b200.varlen.VarlenPlan``): every sequence restarts the covariance,
    states are [N,H]."""
    B, T, H = a.shape
    N.require_cuda(a)
    lib = N.load_library()
    a32, w32, r32, p32 = (x.float().contiguous() for x in (a, omega, r, initial_precision))
    c32 = None if initial_cov is None else initial_cov.float().contiguous()
    gain = torch.empty((B, T, H), dtype=torch.float32, device=a.device)
    p_prev = torch.empty((B, T, H), dtype=torch.float32, device=a.device) if save_state else None
    streams = B if plan is None else plan.num_seqs
    p_final = torch.empty((streams, H), dtype=torch.float32, device=a.device) if want_final else None
    head = (a32.data_ptr(), w32.data_ptr(), r32.data_ptr(), p32.data_ptr(), N.ptr(c32), gain.data_ptr(),
            N.ptr(p_prev), N.ptr(p_final))
    if plan is None:
        ws = N.byte_buffer(lib.kdn_iso_gain_workspace_bytes(B, T, H), a.device)
        N.check(lib.kdn_iso_gain_fwd(*head, B, T, H, float(posterior_scale), ws.data_ptr(), ws.numel(),
                                     N.stream_of(a)), "kdn_iso_gain_fwd")
    else:
        ws = N.byte_buffer(lib.kdn_iso_gain_varlen_workspace_bytes(plan.num_seqs, plan.max_len, H), a.device)
        N.check(lib.kdn_iso_gain_fwd_varlen(*head, T, H, float(posterior_scale), plan.table.data_ptr(),
                                            plan.num_seqs, plan.max_len, ws.data_ptr(), ws.numel(), N.stream_of(a)),
                "kdn_iso_gain_fwd_varlen")
    return gain.to(out_dtype), p_prev, p_final


def _iso_gain_backward(a, omega, r, initial_precision, dgain, p_prev, *, posterior_scale, initial_cov=None,
                       d_final_cov=None, want_d_initial=False, plan=None):
    B, T, H = a.shape
    lib = N.load_library()
    a32, w32, r32, p32, d32 = (x.float().contiguous() for x in (a, omega, r, initial_precision, dgain))
    dfc = None if d_final_cov is None else d_final_cov.float().contiguous()
    da = torch.empty((B, T, H), dtype=torch.float32, device=a.device)
    domega = torch.empty_like(da)
    dr = torch.empty_like(da)
    dinit = torch.empty((H,), dtype=torch.float32, device=a.device)
    streams = B if plan is None else plan.num_seqs
    dic = torch.empty((streams, H), dtype=torch.float32, device=a.device) if want_d_initial else None
    head = (a32.data_ptr(), w32.data_ptr(), r32.data_ptr(), p32.data_ptr(), N.ptr(initial_cov), d32.data_ptr(),
            p_prev.data_ptr(), N.ptr(dfc), da.data_ptr(), domega.data_ptr(), dr.data_ptr(), dinit.data_ptr(),
            N.ptr(dic))
    if plan is None:
        ws = N.byte_buffer(lib.kdn_iso_gain_workspace_bytes(B, T, H), a.device)
        N.check(lib.kdn_iso_gain_bwd(*head, B, T, H, float(posterior_scale), ws.data_ptr(), ws.numel(),
                                     N.stream_of(a)), "kdn_iso_gain_bwd")
    else:
        ws = N.byte_buffer(lib.kdn_iso_gain_varlen_workspace_bytes(plan.num_seqs, plan.max_len, H), a.device)
        N.check(lib.kdn_iso_gain_bwd_varlen(*head, T, H, float(posterior_scale), plan.table.data_ptr(),
                                            plan.num_seqs, plan.max_len, ws.data_ptr(), ws.numel(), N.stream_of(a)),
                "kdn_iso_gain_bwd_varlen")
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
    out_dtype, posterior_scale = _validate_iso_gain_inputs(a, omega, r, initial_precision, head_dim, out_dtype,
                                                           info_scale)
    needs_backward = torch.is_grad_enabled() and any(
        t.requires_grad for t in (a, omega, r, initial_precision)
    )
    return _IsoKDNGainFunction.apply(
        a.contiguous(), omega.contiguous(), r.contiguous(), initial_precision.contiguous(),
        out_dtype, posterior_scale, needs_backward,
    )


def _validate_iso_gain_inputs(a, omega, r, initial_precision, head_dim, out_dtype, info_scale):
    """The reference's checks and messages (iso_kdn_chunk.py:1990-2031);
    returns (out_dtype, posterior_scale = info_scale / head_dim)."""
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
    return out_dtype, posterior_scale


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
    bf16 q/k/v (other floating dtypes are rounded to bf16) with K = V = 128;
    narrower K or V (the reference accepts K <= 256) run zero-padded to 128.
    """
    scale = _validate_chunk_kda_inputs(q, k, v, g_cumsum, beta, scale)
    K, V = q.shape[-1], v.shape[-1]
    if K < 128 or V < 128:
        # narrower heads run in the kernels' 128 channels with zeros above
        # (zero keys and queries keep their norms and leave those state rows
        # at zero, zero values those columns); the pads' backward drops their
        # gradients, the slice's pads the cotangent with zeros
        pk = lambda t: torch.nn.functional.pad(t, (0, 128 - K))  # noqa: E731
        o = _ChunkKDAPrecumsumFunction.apply(pk(q), pk(k), torch.nn.functional.pad(v, (0, 128 - V)),
                                             pk(g_cumsum), beta, scale)
        return o[..., :V]
    return _ChunkKDAPrecumsumFunction.apply(q, k, v, g_cumsum, beta, scale)


def _validate_chunk_kda_inputs(q, k, v, g_cumsum, beta, scale):
    """The reference's checks and messages (iso_kdn_chunk.py:2257-2285) plus
    the kernels' K, V <= 128; returns the scale (K^-0.5 when None)."""
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
    if K > 128 or v.shape[-1] > 128:
        raise ValueError(f"kdn_b200 kernels support K, V <= 128, got K={K}, V={v.shape[-1]}")
    if scale is None:
        scale = K ** -0.5
    return scale


# ----------------------------------------------------------------------------- gate frontend


def _validate_iso_gate_inputs(g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, initial_precision_param,
                              omega_min, r_min):
    """The reference's checks and messages (iso_kdn_chunk.py:1012-1056)."""
    if g_raw.ndim != 4:
        raise ValueError(f"g_raw must have shape [B,T,H,K], got {tuple(g_raw.shape)}")
    B, T, H, K = g_raw.shape
    if K == 0:
        raise ValueError("g_raw's K dimension must be nonzero")
    if omega_r_raw.shape != (B, T, 2 * H):
        raise ValueError(f"omega_r_raw must have shape {(B, T, 2 * H)}, got {tuple(omega_r_raw.shape)}")
    if omega_r_raw.stride(-1) != 1:
        raise ValueError(f"omega_r_raw's head dimension must be contiguous, got strides={omega_r_raw.stride()}")
    for name, value in (("omega_bias", omega_bias), ("r_bias", r_bias)):
        if value.shape != (H,):
            raise ValueError(f"{name} must have shape [{H}], got {tuple(value.shape)}")
    if A_log.shape != (H,):
        raise ValueError(f"A_log must have shape [{H}], got {tuple(A_log.shape)}")
    if dt_bias.shape != (H * K,):
        raise ValueError(f"dt_bias must have shape [{H * K}], got {tuple(dt_bias.shape)}")
    if initial_precision_param.shape != (H,):
        raise ValueError(f"initial_precision_param must have shape [{H}], got {tuple(initial_precision_param.shape)}")
    inputs = (g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, initial_precision_param)
    if not all(value.is_cuda for value in inputs):
        raise ValueError("_iso_kdn_gate_precumsum_paired is a CUDA-only op")
    if any(value.device != g_raw.device for value in inputs[1:]):
        raise ValueError("all scalar-preparation inputs must be on the same CUDA device")
    for name, value in (("g_raw", g_raw), ("omega_r_raw", omega_r_raw)):
        if value.dtype not in (torch.bfloat16, torch.float32):
            raise TypeError(f"{name} must be bf16 or fp32, got {value.dtype}")
    if any(value.dtype != torch.float32 for value in (omega_bias, r_bias, A_log, dt_bias, initial_precision_param)):
        raise TypeError("omega_bias, r_bias, A_log, dt_bias, and initial_precision_param must be FP32")
    for name, value in (("omega_min", omega_min), ("r_min", r_min)):
        if not isinstance(value, (int, float)):
            raise TypeError(f"{name} must be a Python scalar, got {type(value).__name__}")
        if not math.isfinite(float(value)):
            raise ValueError(f"{name} must be finite, got {value!r}")
    if K not in (64, 128):
        raise ValueError(f"g_raw's K dimension must be 64 or 128 on this backend, got {K}")
    return B, T, H, K


def _gate_common(g_raw, omega_r_raw):
    return (g_raw.data_ptr() if g_raw.numel() else None, int(g_raw.dtype == torch.bfloat16),
            omega_r_raw.data_ptr() if omega_r_raw.numel() else None, int(omega_r_raw.dtype == torch.bfloat16),
            omega_r_raw.stride(0), omega_r_raw.stride(1))


def _iso_gate_forward(g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, initial_precision_param, omega_min,
                      r_min):
    B, T, H, K = g_raw.shape
    lib = N.load_library()
    dev = g_raw.device
    g_cumsum = torch.empty((B, T, H, K), dtype=torch.float32, device=dev)
    a = torch.empty((B, T, H), dtype=torch.float32, device=dev)
    omega = torch.empty_like(a)
    r = torch.empty_like(a)
    initial_precision = torch.empty((H,), dtype=torch.float32, device=dev)
    N.check(
        lib.kdn_iso_gate_fwd(
            *_gate_common(g_raw, omega_r_raw), omega_bias.data_ptr(), r_bias.data_ptr(), A_log.data_ptr(),
            dt_bias.data_ptr(), initial_precision_param.data_ptr(), N.ptr(g_cumsum) if g_cumsum.numel() else None,
            N.ptr(a) if a.numel() else None, N.ptr(omega) if a.numel() else None, N.ptr(r) if a.numel() else None,
            initial_precision.data_ptr(), B, T, H, K, float(omega_min), float(r_min), N.stream_of(g_raw),
        ),
        "kdn_iso_gate_fwd",
    )
    return g_cumsum, a, omega, r, initial_precision


def _iso_gate_backward(g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, initial_precision_param,
                       dg_pre_reverse, da, domega, dr, d_initial_precision, needs):
    B, T, H, K = g_raw.shape
    lib = N.load_library()
    (need_dg_raw, need_domega_r_raw, need_domega_bias, need_dr_bias, need_dA_log, need_ddt_bias,
     need_d_param) = needs
    dev = g_raw.device

    def cot(x, shape):
        if x is None:
            return None
        if x.shape != shape:
            raise ValueError(f"cotangent must have shape {shape}, got {tuple(x.shape)}")
        return x.float().contiguous()

    dg_pre_reverse = cot(dg_pre_reverse, (B, T, H, K))
    da, domega, dr = (cot(x, (B, T, H)) for x in (da, domega, dr))
    d_initial_precision = cot(d_initial_precision, (H,))
    dg_raw = torch.empty_like(g_raw) if need_dg_raw else None
    domega_r_raw = torch.empty(omega_r_raw.shape, dtype=omega_r_raw.dtype, device=dev) if need_domega_r_raw else None
    f32 = dict(dtype=torch.float32, device=dev)
    domega_bias = torch.empty((H,), **f32) if need_domega_bias else None
    dr_bias = torch.empty((H,), **f32) if need_dr_bias else None
    dA_log = torch.empty((H,), **f32) if need_dA_log else None
    ddt_bias = torch.empty((H * K,), **f32) if need_ddt_bias else None
    d_param = torch.empty((H,), **f32) if need_d_param else None
    ws = N.byte_buffer(lib.kdn_iso_gate_workspace_bytes(B, T, H, K), dev)
    nz = lambda t: t.data_ptr() if t is not None and t.numel() else None  # noqa: E731
    N.check(
        lib.kdn_iso_gate_bwd(
            *_gate_common(g_raw, omega_r_raw), omega_bias.data_ptr(), r_bias.data_ptr(), A_log.data_ptr(),
            dt_bias.data_ptr(), initial_precision_param.data_ptr(), nz(dg_pre_reverse), nz(da), nz(domega), nz(dr),
            nz(d_initial_precision), nz(dg_raw), nz(domega_r_raw), nz(domega_bias), nz(dr_bias), nz(dA_log),
            nz(ddt_bias), nz(d_param), B, T, H, K, ws.data_ptr(), ws.numel(), N.stream_of(g_raw),
        ),
        "kdn_iso_gate_bwd",
    )
    return dg_raw, domega_r_raw, domega_bias, dr_bias, dA_log, ddt_bias, d_param


class _IsoKDNGatePrecumsumFunction(torch.autograd.Function):
    """Autograd contract of the reference's Function (iso_kdn_chunk.py:1317-1393)."""

    @staticmethod
    def forward(ctx, g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, initial_precision_param, omega_min,
                r_min):
        outs = _iso_gate_forward(g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, initial_precision_param,
                                 omega_min, r_min)
        ctx.save_for_backward(g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, initial_precision_param)
        ctx.set_materialize_grads(False)
        return outs

    @staticmethod
    def backward(ctx, dg_pre_reverse, da, domega, dr, d_initial_precision):
        g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, param = ctx.saved_tensors
        grads = _iso_gate_backward(g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, param, dg_pre_reverse,
                                   da, domega, dr, d_initial_precision, ctx.needs_input_grad[:7])
        return (*grads, None, None)


@torch.compiler.disable
def _iso_kdn_gate_precumsum_paired(
    g_raw: torch.Tensor,
    omega_r_raw: torch.Tensor,
    omega_bias: torch.Tensor,
    r_bias: torch.Tensor,
    A_log: torch.Tensor,
    dt_bias: torch.Tensor,
    initial_precision_param: torch.Tensor,
    omega_min: float,
    r_min: float,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Return the paired ``(base2_prefix, a, omega, r, initial_precision)`` tensors
    (iso_kdn_chunk.py:1396-1431).

    ``base2_prefix`` (the 64-token-chunk-local base-2 gate prefix) must have
    exactly one consumer, ``_chunk_kda_precumsum_paired``: the two Functions
    exchange the gate cotangent in natural-log coordinates before the reverse
    prefix sum, not a generic tensor VJP.
    """
    _validate_iso_gate_inputs(g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, initial_precision_param,
                              omega_min, r_min)
    return _IsoKDNGatePrecumsumFunction.apply(
        g_raw.contiguous(), omega_r_raw, omega_bias.contiguous(), r_bias.contiguous(), A_log.contiguous(),
        dt_bias.contiguous(), initial_precision_param.contiguous(), float(omega_min), float(r_min),
    )


__all__ = ("_chunk_kda_precumsum_paired", "_iso_kdn_gate_precumsum_paired", "iso_kdn_gain")
