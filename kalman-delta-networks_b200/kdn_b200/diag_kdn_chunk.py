"""Diagonal KDN operators on B200: drop-in replacements for

* ``_diag_kdn_gain`` (lit_gpt/kdn_ops/diag_kdn_chunk.py:2737)
* ``chunk_kalman``   (lit_gpt/kdn_ops/diag_kdn_chunk.py:3315)
* ``_diag_kdn_frontend_precumsum_paired`` (lit_gpt/kdn_ops/diag_kdn_chunk.py:2471)
* ``_diag_kdn_normalize`` (lit_gpt/kdn_ops/diag_kdn_chunk.py:2162)

with the reference's signatures, validation messages, tensor layouts and
autograd contract, on the sm_100a kernels of ``libkdn_b200.so``.
"""
from __future__ import annotations

import math

import torch
from torch.autograd.function import once_differentiable

from . import _native as N
from ._scan import ScanSaved, scan_backward, scan_forward

_VECTOR_DTYPE = torch.bfloat16
_STATE_DTYPE = torch.float32
_KD = 128  # the kernels' key and value width


def _gain_forward(k, alpha, omega, r, initial_precision, initial_cov=None, want_final=False, plan=None):
    """Forward per-channel covariance scan; optional carried-in covariance
    [B,H,K] and final covariance out (sequence parallelism).  ``plan`` (a
    packed batch's ``kdn_b200.varlen.VarlenPlan``): every sequence restarts
    the covariance, states are [N,H,K]."""
    B, T, H, K = k.shape
    N.require_cuda(k)
    lib = N.load_library()
    kappa = torch.empty_like(k, dtype=_STATE_DTYPE)
    streams = B if plan is None else plan.num_seqs
    p_final = torch.empty((streams, H, K), dtype=torch.float32, device=k.device) if want_final else None
    if plan is None:
        carry = torch.empty(lib.kdn_diag_gain_carry_elems(B, T, H, K), dtype=torch.float32, device=k.device)
        ws = N.byte_buffer(lib.kdn_diag_gain_workspace_bytes(B, T, H, K), k.device)
        N.check(
            lib.kdn_diag_gain_fwd(
                k.data_ptr(), alpha.data_ptr(), omega.data_ptr(), r.data_ptr(), initial_precision.data_ptr(),
                N.ptr(initial_cov), kappa.data_ptr(), carry.data_ptr(), N.ptr(p_final), B, T, H, K, ws.data_ptr(),
                ws.numel(), N.stream_of(k),
            ),
            "kdn_diag_gain_fwd",
        )
    else:
        nc = plan.num_chunks
        carry = torch.empty(lib.kdn_diag_gain_varlen_carry_elems(T, H, K, nc), dtype=torch.float32, device=k.device)
        ws = N.byte_buffer(lib.kdn_diag_gain_varlen_workspace_bytes(T, H, K, nc), k.device)
        N.check(
            lib.kdn_diag_gain_fwd_varlen(
                k.data_ptr(), alpha.data_ptr(), omega.data_ptr(), r.data_ptr(), initial_precision.data_ptr(),
                N.ptr(initial_cov), kappa.data_ptr(), carry.data_ptr(), N.ptr(p_final), T, H, K,
                plan.table.data_ptr(), plan.num_seqs, nc, ws.data_ptr(), ws.numel(), N.stream_of(k),
            ),
            "kdn_diag_gain_fwd_varlen",
        )
    return kappa, carry, p_final


def _gain_backward(k, alpha, omega, r, initial_precision, omega_raw, r_raw, dkappa, carry, need_initial,
                   initial_cov=None, d_final_cov=None, want_d_initial=False, plan=None):
    B, T, H, K = k.shape
    lib = N.load_library()
    dkappa = torch.zeros_like(k) if dkappa is None else dkappa.float().contiguous()
    dk = torch.empty_like(k, dtype=_STATE_DTYPE)
    dalpha = torch.empty_like(alpha, dtype=_STATE_DTYPE)
    domega_raw = torch.empty_like(omega_raw)
    dr_raw = torch.empty_like(r_raw)
    dinit = torch.empty((H,), dtype=_STATE_DTYPE, device=k.device) if need_initial else None
    streams = B if plan is None else plan.num_seqs
    dic = torch.empty((streams, H, K), dtype=_STATE_DTYPE, device=k.device) if want_d_initial else None
    dfc = None if d_final_cov is None else d_final_cov.float().contiguous()
    head = (k.data_ptr(), alpha.data_ptr(), omega.data_ptr(), r.data_ptr(), initial_precision.data_ptr(),
            N.ptr(initial_cov), omega_raw.data_ptr(), r_raw.data_ptr(), dkappa.data_ptr(), carry.data_ptr(),
            N.ptr(dfc), dk.data_ptr(), dalpha.data_ptr(), domega_raw.data_ptr(), dr_raw.data_ptr(), N.ptr(dinit),
            N.ptr(dic))
    if plan is None:
        ws = N.byte_buffer(lib.kdn_diag_gain_workspace_bytes(B, T, H, K), k.device)
        N.check(lib.kdn_diag_gain_bwd(*head, B, T, H, K, ws.data_ptr(), ws.numel(), N.stream_of(k)),
                "kdn_diag_gain_bwd")
    else:
        nc = plan.num_chunks
        ws = N.byte_buffer(lib.kdn_diag_gain_varlen_workspace_bytes(T, H, K, nc), k.device)
        N.check(lib.kdn_diag_gain_bwd_varlen(*head, T, H, K, plan.table.data_ptr(), plan.num_seqs, nc,
                                             ws.data_ptr(), ws.numel(), N.stream_of(k)),
                "kdn_diag_gain_bwd_varlen")
    return dk, dalpha, domega_raw, dr_raw, dinit, dic


class _DiagKdnGainFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, k, alpha, omega, r, initial_precision, omega_raw, r_raw):
        kappa, carry, _ = _gain_forward(k, alpha, omega, r, initial_precision)
        ctx.save_for_backward(k, alpha, omega, r, initial_precision, omega_raw, r_raw, carry)
        ctx.set_materialize_grads(False)
        return kappa

    @staticmethod
    @once_differentiable
    def backward(ctx, dkappa):
        k, alpha, omega, r, initial_precision, omega_raw, r_raw, carry = ctx.saved_tensors
        needs = ctx.needs_input_grad
        dk, dalpha, domega_raw, dr_raw, dinit, _ = _gain_backward(
            k, alpha, omega, r, initial_precision, omega_raw, r_raw, dkappa, carry, need_initial=needs[4]
        )
        return (
            dk if needs[0] else None,
            dalpha if needs[1] else None,
            None,
            None,
            dinit if needs[4] else None,
            domega_raw if needs[5] else None,
            dr_raw if needs[6] else None,
        )


def _diag_kdn_gain(k_gain, alpha, omega, r, initial_precision, omega_raw, r_raw):
    """Fixed-scale FP32 diagonal gain with fused raw-logit VJPs (diag_kdn_chunk.py:2737-2791)."""
    _validate_diag_kdn_gain_inputs(k_gain, alpha, omega, r, initial_precision, omega_raw, r_raw)
    return _DiagKdnGainFunction.apply(
        k_gain, alpha, omega.detach(), r.detach(), initial_precision, omega_raw, r_raw
    )


def _validate_diag_kdn_gain_inputs(k_gain, alpha, omega, r, initial_precision, omega_raw, r_raw):
    """The reference's checks and messages (diag_kdn_chunk.py:2747-2791); returns (B, T, H, K)."""
    tensors = {
        "k_gain": k_gain,
        "alpha": alpha,
        "omega": omega,
        "r": r,
        "initial_precision": initial_precision,
        "omega_raw": omega_raw,
        "r_raw": r_raw,
    }
    for name, value in tensors.items():
        if not isinstance(value, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if not value.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if value.device != k_gain.device:
            raise ValueError("all DiagKDN gain inputs must share one CUDA device")
        if not value.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if k_gain.ndim != 4:
        raise ValueError("k_gain must have rank 4 [B,T,H,K]")
    B, T, H, K = k_gain.shape
    if min(B, T, H) <= 0 or K not in (64, 128):
        raise ValueError("DiagKDN gain requires non-empty B/T/H and K in {64,128}")
    expected = (B, T, H, K)
    for name in ("alpha", "omega", "omega_raw"):
        if tensors[name].shape != expected:
            raise ValueError(f"{name} must have shape {expected}")
    if r.shape != (B, T, H) or r_raw.shape != (B, T, H):
        raise ValueError("r and r_raw must have shape [B,T,H]")
    if initial_precision.shape != (H,):
        raise ValueError(f"initial_precision must have shape [{H}]")
    for name in ("k_gain", "alpha", "omega", "r", "initial_precision"):
        if tensors[name].dtype != torch.float32:
            raise TypeError(f"{name} must be torch.float32")
    if omega_raw.dtype != _VECTOR_DTYPE or r_raw.dtype != _VECTOR_DTYPE:
        raise TypeError("omega_raw and r_raw must be torch.bfloat16")
    return B, T, H, K


def _validate_diag_kdn_memory_inputs(q, k, kappa, v, g_cumsum, scale):
    tensors = {"q": q, "k": k, "kappa": kappa, "v": v, "g_cumsum": g_cumsum}
    for name, value in tensors.items():
        if not isinstance(value, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if value.ndim != 4:
            raise ValueError(f"{name} must have rank 4 [B,T,H,D]")
        if not value.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if value.device != q.device:
            raise ValueError("all DiagKDN memory inputs must share one CUDA device")
        if not value.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    B, T, H, K = q.shape
    if min(B, T, H) <= 0 or K not in (64, 128):
        raise ValueError("DiagKDN memory requires non-empty B/T/H and K in {64,128}")
    expected = (B, T, H, K)
    for name in ("k", "kappa", "v", "g_cumsum"):
        if tensors[name].shape != expected:
            raise ValueError(f"{name} must have shape {expected}")
    for name in ("q", "k", "v"):
        if tensors[name].dtype != _VECTOR_DTYPE:
            raise TypeError(f"{name} must be torch.bfloat16")
    if kappa.dtype != _STATE_DTYPE or g_cumsum.dtype != _STATE_DTYPE:
        raise TypeError("kappa and g_cumsum must be torch.float32")
    if type(scale) is not float or not math.isfinite(scale):
        raise TypeError("scale must be an exact finite float")
    return B, T, H, K


class _DiagKdnMemoryFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, kappa, v, g_cumsum, scale):
        output, _, saved = scan_forward(N.KDN_DIAG, q, k, v, g_cumsum, kappa, scale)
        ctx.save_for_backward(q, k, kappa, v, g_cumsum, saved.saved)
        ctx.precision = saved.precision
        ctx.scale = scale
        ctx.set_materialize_grads(False)
        return output

    @staticmethod
    @once_differentiable
    def backward(ctx, do):
        q, k, kappa, v, g_cumsum, saved = ctx.saved_tensors
        if do is None:
            return None, None, None, None, None, None
        do = do.contiguous()
        B, T, H, K = _validate_diag_kdn_memory_inputs(q, k, kappa, v, g_cumsum, ctx.scale)
        if do.shape != (B, T, H, K) or do.dtype != torch.float32:
            raise TypeError("DiagKDN output cotangent must be FP32 BTHK")
        dq, dk, dv, dG, dkappa, _ = scan_backward(
            N.KDN_DIAG, q, k, v, g_cumsum, kappa, ctx.scale, ScanSaved(saved, ctx.precision), do
        )
        return dq, dk, dkappa, dv, dG, None


def chunk_kalman(
    q_memory: torch.Tensor,
    k_memory: torch.Tensor,
    kappa: torch.Tensor,
    v: torch.Tensor,
    g_cumsum: torch.Tensor,
    scale: float,
) -> torch.Tensor:
    """Diagonal KDN memory scan (diag_kdn_chunk.py:3315-3332): fp32 output;
    backward returns (dq bf16, dk bf16, dkappa fp32, dv bf16, dG fp32, None)
    with dG the natural-log cotangent before the reverse 32-chunk cumsum.
    K = V in {64, 128}, as the reference (64 runs zero-padded to 128)."""
    K = _validate_diag_kdn_memory_inputs(q_memory, k_memory, kappa, v, g_cumsum, scale)[3]
    if K < _KD:
        # K = V = 64: the kernels' 128 channels with zeros in the upper half
        # (zero keys, gains and values leave those state rows and columns at
        # zero and add nothing to any product); the pads' backward drops
        # their gradients, the slice's pads the cotangent with zeros
        pad = lambda t: torch.nn.functional.pad(t, (0, _KD - K))  # noqa: E731
        o = _DiagKdnMemoryFunction.apply(pad(q_memory), pad(k_memory), pad(kappa), pad(v), pad(g_cumsum), scale)
        return o[..., :K]
    return _DiagKdnMemoryFunction.apply(q_memory, k_memory, kappa, v, g_cumsum, scale)


# --------------------------------------------------------------------------
# Gate / noise frontend


def _validate_diag_kdn_frontend_inputs(retention_raw, omega_raw, r_raw, A_log, dt_bias, initial_precision_param):
    """The reference's checks and messages (diag_kdn_chunk.py:2171-2215)."""
    tensors = {
        "retention_raw": retention_raw,
        "omega_raw": omega_raw,
        "r_raw": r_raw,
        "A_log": A_log,
        "dt_bias": dt_bias,
        "initial_precision_param": initial_precision_param,
    }
    for name, value in tensors.items():
        if not isinstance(value, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if not value.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if value.device != retention_raw.device:
            raise ValueError("all DiagKDN frontend inputs must share one CUDA device")
        if not value.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if retention_raw.ndim != 4:
        raise ValueError("retention_raw must have rank 4 [B,T,H,K]")
    B, T, H, K = retention_raw.shape
    if min(B, T, H) <= 0 or K not in (64, 128):
        raise ValueError("DiagKDN frontend requires non-empty B/T/H and K in {64,128}")
    if omega_raw.shape != (B, T, H, K):
        raise ValueError("omega_raw must match retention_raw")
    if r_raw.shape != (B, T, H):
        raise ValueError("r_raw must have shape [B,T,H]")
    if A_log.shape != (H,) or initial_precision_param.shape != (H,):
        raise ValueError("A_log and initial_precision_param must have shape [H]")
    if dt_bias.shape != (H, K):
        raise ValueError("dt_bias must have shape [H,K]")
    for name in ("retention_raw", "omega_raw", "r_raw"):
        if tensors[name].dtype != _VECTOR_DTYPE:
            raise TypeError(f"{name} must be torch.bfloat16")
    for name in ("A_log", "dt_bias", "initial_precision_param"):
        if tensors[name].dtype != _STATE_DTYPE:
            raise TypeError(f"{name} must be torch.float32")
    return B, T, H, K


def _diag_frontend_forward(retention_raw, omega_raw, r_raw, A_log, dt_bias, initial_precision_param):
    B, T, H, K = retention_raw.shape
    lib = N.load_library()
    dev = retention_raw.device
    g_cumsum = torch.empty((B, T, H, K), dtype=_STATE_DTYPE, device=dev)
    alpha = torch.empty_like(g_cumsum)
    omega = torch.empty_like(g_cumsum)
    r = torch.empty((B, T, H), dtype=_STATE_DTYPE, device=dev)
    initial_precision = torch.empty((H,), dtype=_STATE_DTYPE, device=dev)
    N.check(
        lib.kdn_diag_gate_fwd(
            retention_raw.data_ptr(), omega_raw.data_ptr(), r_raw.data_ptr(), A_log.data_ptr(), dt_bias.data_ptr(),
            initial_precision_param.data_ptr(), g_cumsum.data_ptr(), alpha.data_ptr(), omega.data_ptr(),
            r.data_ptr(), initial_precision.data_ptr(), B, T, H, K, N.stream_of(retention_raw),
        ),
        "kdn_diag_gate_fwd",
    )
    return g_cumsum, alpha, omega, r, initial_precision


def _diag_frontend_backward(retention_raw, omega_raw, r_raw, A_log, dt_bias, initial_precision_param, d_g_cumsum,
                            d_alpha, d_omega, d_r, d_initial_precision, needs):
    """Gradients for the inputs in ``needs`` whose cotangents are present, None
    for the others (diag_kdn_chunk.py:2265-2443)."""
    B, T, H, K = retention_raw.shape
    lib = N.load_library()
    dev = retention_raw.device
    need_retention, need_omega, need_r, need_A, need_dt, need_initial = needs

    def cot(x, shape):
        if x is None:
            return None
        if x.shape != shape:
            raise ValueError(f"cotangent must have shape {shape}, got {tuple(x.shape)}")
        return x.to(_STATE_DTYPE).contiguous()

    d_g_cumsum, d_alpha, d_omega = (cot(x, (B, T, H, K)) for x in (d_g_cumsum, d_alpha, d_omega))
    d_r = cot(d_r, (B, T, H))
    d_initial_precision = cot(d_initial_precision, (H,))
    has_decay = d_g_cumsum is not None or d_alpha is not None
    f32 = dict(dtype=_STATE_DTYPE, device=dev)
    dretention_raw = torch.empty_like(retention_raw) if has_decay and need_retention else None
    dA_log = torch.empty((H,), **f32) if has_decay and need_A else None
    ddt_bias = torch.empty((H, K), **f32) if has_decay and need_dt else None
    domega_raw = torch.empty_like(omega_raw) if need_omega and d_omega is not None else None
    dr_raw = torch.empty_like(r_raw) if need_r and d_r is not None else None
    d_param = torch.empty((H,), **f32) if need_initial and d_initial_precision is not None else None
    ws = N.byte_buffer(lib.kdn_diag_gate_workspace_bytes(B, T, H, K), dev)
    N.check(
        lib.kdn_diag_gate_bwd(
            retention_raw.data_ptr(), omega_raw.data_ptr(), r_raw.data_ptr(), A_log.data_ptr(), dt_bias.data_ptr(),
            initial_precision_param.data_ptr(), N.ptr(d_g_cumsum), N.ptr(d_alpha), N.ptr(d_omega), N.ptr(d_r),
            N.ptr(d_initial_precision), N.ptr(dretention_raw), N.ptr(domega_raw), N.ptr(dr_raw), N.ptr(dA_log),
            N.ptr(ddt_bias), N.ptr(d_param), B, T, H, K, ws.data_ptr(), ws.numel(), N.stream_of(retention_raw),
        ),
        "kdn_diag_gate_bwd",
    )
    return dretention_raw, domega_raw, dr_raw, dA_log, ddt_bias, d_param


class _DiagKdnFrontendFunction(torch.autograd.Function):
    """Autograd contract of the reference's Function (diag_kdn_chunk.py:2446-2468)."""

    @staticmethod
    def forward(ctx, retention_raw, omega_raw, r_raw, A_log, dt_bias, initial_precision_param):
        outs = _diag_frontend_forward(retention_raw, omega_raw, r_raw, A_log, dt_bias, initial_precision_param)
        # alpha is recomputed from retention_raw in the backward kernel
        ctx.save_for_backward(retention_raw, omega_raw, r_raw, A_log, dt_bias, initial_precision_param)
        ctx.set_materialize_grads(False)
        return outs

    @staticmethod
    @once_differentiable
    def backward(ctx, d_g_cumsum, d_alpha, d_omega, d_r, d_initial_precision):
        return _diag_frontend_backward(*ctx.saved_tensors, d_g_cumsum, d_alpha, d_omega, d_r, d_initial_precision,
                                       ctx.needs_input_grad)


def _diag_kdn_frontend_precumsum_paired(
    retention_raw: torch.Tensor,
    omega_raw: torch.Tensor,
    r_raw: torch.Tensor,
    A_log: torch.Tensor,
    dt_bias: torch.Tensor,
    initial_precision_param: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Apply the fixed uncoupled omega=0 / r=0.01 32-token frontend
    (diag_kdn_chunk.py:2471-2494): returns ``(g_cumsum, alpha, omega, r,
    initial_precision)``.

    ``g_cumsum`` (the chunk-local base-2 prefix of ln max(alpha, 1e-6)) is
    paired with its consumer: the cotangent it receives is reverse-prefixed in
    natural-log coordinates, without the log2(e) factor.
    """
    _validate_diag_kdn_frontend_inputs(retention_raw, omega_raw, r_raw, A_log, dt_bias, initial_precision_param)
    return _DiagKdnFrontendFunction.apply(retention_raw, omega_raw, r_raw, A_log, dt_bias, initial_precision_param)


# ----------------------------------------------------------------------------- q / k normalisation


def _validate_diag_kdn_norm_inputs(q_raw, k_raw):
    """The reference's checks and messages (diag_kdn_chunk.py:2024-2042)."""
    for name, value in (("q_raw", q_raw), ("k_raw", k_raw)):
        if not isinstance(value, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if value.ndim != 4:
            raise ValueError(f"{name} must have rank 4 [B,T,H,K]")
        if not value.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if value.dtype not in (torch.bfloat16, torch.float32):
            raise TypeError(f"{name} must be BF16 or FP32")
        if not value.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if q_raw.shape != k_raw.shape or q_raw.device != k_raw.device:
        raise ValueError("q_raw and k_raw must have matching shape and device")
    if q_raw.dtype != k_raw.dtype or q_raw.requires_grad != k_raw.requires_grad:
        raise ValueError("q_raw and k_raw must have matching dtype and grad mode")
    if q_raw.shape[-1] not in (64, 128):
        raise ValueError("q_raw and k_raw require K in {64,128}")


class _DiagKdnNormFunction(torch.autograd.Function):
    """(q_memory bf16, k_gain fp32, k_memory bf16) = the rows of q and k over
    their L2 norms (kdn_diag_norm_fwd); the norms are saved for the backward
    (kdn_diag_norm_bwd).  Absent cotangents stay absent, as in the
    reference's Function (diag_kdn_chunk.py:2045-2075)."""

    @staticmethod
    def forward(ctx, q_raw, k_raw):
        N.require_cuda(q_raw, k_raw)
        lib = N.load_library()
        K = q_raw.shape[-1]
        rows = q_raw.numel() // K
        q_memory = torch.empty(q_raw.shape, dtype=torch.bfloat16, device=q_raw.device)
        k_gain = torch.empty(k_raw.shape, dtype=torch.float32, device=k_raw.device)
        k_memory = torch.empty(k_raw.shape, dtype=torch.bfloat16, device=k_raw.device)
        q_norm = torch.empty(q_raw.shape[:-1], dtype=torch.float32, device=q_raw.device)
        k_norm = torch.empty(k_raw.shape[:-1], dtype=torch.float32, device=k_raw.device)
        N.check(lib.kdn_diag_norm_fwd(q_raw.data_ptr(), k_raw.data_ptr(), int(q_raw.dtype == torch.bfloat16),
                                      q_memory.data_ptr(), k_gain.data_ptr(), k_memory.data_ptr(), q_norm.data_ptr(),
                                      k_norm.data_ptr(), rows, K, N.stream_of(q_raw)), "kdn_diag_norm_fwd")
        ctx.save_for_backward(q_raw, k_raw, q_norm, k_norm)
        ctx.set_materialize_grads(False)
        return q_memory, k_gain, k_memory

    @staticmethod
    @once_differentiable
    def backward(ctx, d_q_memory, d_k_gain, d_k_memory):
        if not ctx.needs_input_grad[0]:
            d_q_memory = None
        if not ctx.needs_input_grad[1]:
            d_k_gain = d_k_memory = None
        if d_q_memory is None and d_k_gain is None and d_k_memory is None:
            return None, None
        q_raw, k_raw, q_norm, k_norm = ctx.saved_tensors
        lib = N.load_library()
        K = q_raw.shape[-1]
        rows = q_raw.numel() // K
        dqm = None if d_q_memory is None else d_q_memory.to(torch.bfloat16).contiguous()
        dkg = None if d_k_gain is None else d_k_gain.float().contiguous()
        dkm = None if d_k_memory is None else d_k_memory.to(torch.bfloat16).contiguous()
        dq = torch.empty_like(q_raw) if dqm is not None else None
        dk = torch.empty_like(k_raw) if (dkg is not None or dkm is not None) else None
        N.check(lib.kdn_diag_norm_bwd(q_raw.data_ptr(), k_raw.data_ptr(), int(q_raw.dtype == torch.bfloat16),
                                      N.ptr(dqm), N.ptr(dkg), N.ptr(dkm), q_norm.data_ptr(), k_norm.data_ptr(),
                                      N.ptr(dq), N.ptr(dk), rows, K, N.stream_of(q_raw)), "kdn_diag_norm_bwd")
        return dq, dk


def _diag_kdn_normalize(q_raw, k_raw):
    """Normalise q and k at the diagonal mixer's bf16 boundary: returns
    ``(q_memory bf16, k_gain fp32, k_memory bf16)``, bit-identical to the
    reference (its rounding steps and reduction order, see
    ``csrc/kdn_norm.cu``).  Replaces diag_kdn_chunk.py:2162."""
    _validate_diag_kdn_norm_inputs(q_raw, k_raw)
    return _DiagKdnNormFunction.apply(q_raw, k_raw)


__all__ = ("_diag_kdn_gain", "chunk_kalman", "_diag_kdn_frontend_precumsum_paired", "_diag_kdn_normalize")
