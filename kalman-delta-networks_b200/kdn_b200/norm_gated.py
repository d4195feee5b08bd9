"""Gated RMS normalisation of the scan output on B200: a drop-in for
flash-linear-attention's ``FusedRMSNormGated`` / ``rms_norm_gated``
(fla.modules.fused_norm_gate), which both reference mixers apply to the scan
output before the output projection (lit_gpt/iso_kdn.py:192-197, 305-314;
lit_gpt/diag_kdn.py:216-221, 346-355: activation "sigmoid", one row per head
of ``head_v_dim``).

    y = x / sqrt(mean(x^2) + eps) * weight * act(g),  act = sigmoid or g * sigmoid(g)

Same constructor, forward signature, parameter and output dtypes; the
kernels (``kdn_rmsnorm_gated_fwd`` / ``_bwd`` of ``libkdn_b200.so``) compute
in fp32.  Rows are the last axis (64 or 128 wide); the residual / prenorm
options of the flash-linear-attention module, which the mixers do not use,
are not supported (they raise).
"""
from __future__ import annotations

import torch
import torch.nn as nn
from torch.autograd.function import once_differentiable

from . import _native as N

_ACTIVATIONS = {"sigmoid": 0, "swish": 1, "silu": 1}


class _RMSNormGatedFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, g, weight, activation, eps):
        N.require_cuda(x, g)
        lib = N.load_library()
        D = x.shape[-1]
        xs, gs = x.contiguous(), g.contiguous()
        rows = xs.numel() // D
        y = torch.empty_like(xs)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        w = None if weight is None else weight.float().contiguous()
        N.check(lib.kdn_rmsnorm_gated_fwd(xs.data_ptr(), int(xs.dtype == torch.bfloat16), gs.data_ptr(),
                                          int(gs.dtype == torch.bfloat16), N.ptr(w), y.data_ptr(), rstd.data_ptr(),
                                          rows, D, float(eps), _ACTIVATIONS[activation], N.stream_of(xs)),
                "kdn_rmsnorm_gated_fwd")
        ctx.save_for_backward(xs, gs, w, rstd)
        ctx.meta = (activation, weight is not None, None if weight is None else weight.dtype, x.shape, g.shape)
        return y.view(x.shape)

    @staticmethod
    @once_differentiable
    def backward(ctx, dy):
        xs, gs, w, rstd = ctx.saved_tensors
        activation, has_w, w_dtype, x_shape, g_shape = ctx.meta
        lib = N.load_library()
        D = xs.shape[-1]
        rows = xs.numel() // D
        dy = dy.to(xs.dtype).contiguous()
        dx, dg = torch.empty_like(xs), torch.empty_like(gs)
        dw = torch.empty(D, dtype=torch.float32, device=xs.device) if has_w and ctx.needs_input_grad[2] else None
        ws = N.byte_buffer(lib.kdn_rmsnorm_gated_workspace_bytes(rows, D), xs.device) if dw is not None else None
        N.check(lib.kdn_rmsnorm_gated_bwd(xs.data_ptr(), int(xs.dtype == torch.bfloat16), gs.data_ptr(),
                                          int(gs.dtype == torch.bfloat16), N.ptr(w), dy.data_ptr(), rstd.data_ptr(),
                                          dx.data_ptr(), dg.data_ptr(), N.ptr(dw), rows, D,
                                          _ACTIVATIONS[activation], N.ptr(ws), 0 if ws is None else ws.numel(),
                                          N.stream_of(xs)), "kdn_rmsnorm_gated_bwd")
        return dx.view(x_shape), dg.view(g_shape), None if dw is None else dw.to(w_dtype), None, None


def rms_norm_gated(x, g, weight, bias=None, activation="swish", residual=None, prenorm=False,
                   residual_in_fp32=False, eps=1e-6):
    """Functional form, flash-linear-attention's ``rms_norm_gated`` signature."""
    if bias is not None or residual is not None or prenorm or residual_in_fp32:
        raise NotImplementedError("kdn_b200 rms_norm_gated: bias, residual and prenorm are not supported")
    if activation not in _ACTIVATIONS:
        raise ValueError(f"Unsupported activation: {activation}")
    if x.shape != g.shape:
        raise ValueError("x and g must have the same shape")
    if x.shape[-1] not in (64, 128):
        raise ValueError("kdn_b200 rms_norm_gated: the normalised width must be 64 or 128")
    if x.dtype not in (torch.bfloat16, torch.float32) or g.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("kdn_b200 rms_norm_gated: x and g must be bf16 or fp32")
    if weight is not None and weight.shape != (x.shape[-1],):
        raise ValueError("weight must have shape [D]")
    return _RMSNormGatedFunction.apply(x, g, weight, activation, eps)


class FusedRMSNormGated(nn.Module):
    """Drop-in for ``fla.modules.FusedRMSNormGated`` (same constructor, same
    ``weight`` parameter initialised to ones, same forward signature)."""

    def __init__(self, hidden_size, elementwise_affine=True, eps=1e-5, activation="swish", device=None,
                 dtype=None):
        super().__init__()
        self.hidden_size = hidden_size
        self.elementwise_affine = elementwise_affine
        self.eps = eps
        self.activation = activation
        if self.activation not in ["swish", "silu", "sigmoid"]:
            raise ValueError(f"Unsupported activation: {self.activation}")
        if elementwise_affine:
            self.weight = nn.Parameter(torch.empty(hidden_size, device=device, dtype=dtype))
        else:
            self.register_parameter("weight", None)
        self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self):
        if self.elementwise_affine:
            nn.init.ones_(self.weight)

    def forward(self, x, g, residual=None, prenorm=False, residual_in_fp32=False):
        return rms_norm_gated(x, g, self.weight, self.bias, self.activation, residual=residual, eps=self.eps,
                              prenorm=prenorm, residual_in_fp32=residual_in_fp32)


__all__ = ("FusedRMSNormGated", "rms_norm_gated")
