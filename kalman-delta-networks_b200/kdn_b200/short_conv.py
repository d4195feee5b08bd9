"""Short causal depthwise convolution with SiLU on B200: the convolution the
mixers apply to their q, k, v projections before the scan.

* ``qkv_causal_conv1d(x, weight)`` replaces the packed one of the isotropic
  mixer (lit_gpt/kdn_ops/iso_kdn_chunk.py:459, Function :431; called by
  ``PackedQKV.forward``, :575): x [B, T, 3D] packed q|k|v channels, weight
  [3D, 4] -> (q, k, v), each [B, T, D].  Same validation messages.
* ``fixed_short_conv(convolution, hidden_states)`` replaces
  ``_fixed_short_conv`` of the diagonal mixer (lit_gpt/diag_kdn.py:75, which
  calls flash-linear-attention's ``causal_conv1d`` with SiLU): one tensor
  [B, T, D] with the depthwise ``nn.Conv1d`` weight [D, 1, 4].

    y[b, t, c] = silu(sum_j w[c, j] x[b, t - 3 + j, c])   (x = 0 before t = 0)

The kernels (``kdn_short_conv_fwd`` / ``_bwd``) compute in fp32; outputs and
the input gradient take x's dtype, the weight gradient the weight's.  The
projection in front (``F.linear``) is a plain GEMM and stays with cuBLAS.
"""
from __future__ import annotations

import ctypes

import torch
from torch.autograd.function import once_differentiable

from . import _native as N

KERNEL_WIDTH = 4
GROUPS = 3


def _validate_qkv_conv_inputs(x, weight):
    """The reference's checks and messages (iso_kdn_chunk.py:255-278)."""
    if x.ndim != 3:
        raise ValueError(f"packed input must be rank-3 [B,T,3D], got {tuple(x.shape)}")
    if x.shape[0] < 1 or x.shape[1] < 1:
        raise ValueError(f"batch and sequence dimensions must be positive, got {tuple(x.shape)}")
    packed_width = x.shape[-1]
    if packed_width < GROUPS or packed_width % GROUPS != 0:
        raise ValueError(f"packed input width must be a positive multiple of {GROUPS}, got {packed_width}")
    if weight.shape != (packed_width, KERNEL_WIDTH):
        raise ValueError(f"packed weight must be [{packed_width},{KERNEL_WIDTH}], got {tuple(weight.shape)}")
    if x.device.type != "cuda" or weight.device != x.device:
        raise ValueError("QKV causal convolution requires colocated CUDA tensors")
    allowed_dtypes = (torch.bfloat16, torch.float32)
    if x.dtype not in allowed_dtypes:
        raise TypeError(f"packed input must be bfloat16 or float32, got {x.dtype}")
    if weight.dtype not in allowed_dtypes:
        raise TypeError(f"packed weight must be bfloat16 or float32, got {weight.dtype}")
    if not x.is_contiguous() or not weight.is_contiguous():
        raise ValueError("packed input and weight must already be contiguous")
    return packed_width // GROUPS


class _ShortConv(torch.autograd.Function):
    """groups outputs [B, T, C / groups] from x [B, T, C] and weight [C, 4]."""

    @staticmethod
    def forward(ctx, x, weight, groups):
        N.require_cuda(x, weight)
        lib = N.load_library()
        B, T, C = x.shape
        D = C // groups
        if D % 2:
            raise ValueError("kdn_b200 short convolution: channels per tensor must be even")
        ys = [torch.empty(B, T, D, dtype=x.dtype, device=x.device) for _ in range(groups)]
        ptrs = (ctypes.c_void_p * 3)(*[y.data_ptr() for y in ys], *([None] * (3 - groups)))
        N.check(lib.kdn_short_conv_fwd(x.data_ptr(), int(x.dtype == torch.bfloat16), weight.data_ptr(),
                                       int(weight.dtype == torch.bfloat16), ptrs, groups, B, T, C, KERNEL_WIDTH, 1,
                                       N.stream_of(x)), "kdn_short_conv_fwd")
        ctx.save_for_backward(x, weight)
        ctx.groups = groups
        ctx.set_materialize_grads(False)
        return tuple(ys)

    @staticmethod
    @once_differentiable
    def backward(ctx, *dys):
        x, weight = ctx.saved_tensors
        if all(d is None for d in dys):
            return None, None, None
        lib = N.load_library()
        B, T, C = x.shape
        dys = [None if d is None else d.to(x.dtype).contiguous() for d in dys]
        ptrs = (ctypes.c_void_p * 3)(*[N.ptr(d) for d in dys], *([None] * (3 - ctx.groups)))
        dx, dw = torch.empty_like(x), torch.empty_like(weight)
        ws = N.byte_buffer(lib.kdn_short_conv_workspace_bytes(B, T, C, KERNEL_WIDTH), x.device)
        N.check(lib.kdn_short_conv_bwd(x.data_ptr(), int(x.dtype == torch.bfloat16), weight.data_ptr(),
                                       int(weight.dtype == torch.bfloat16), ptrs, ctx.groups, dx.data_ptr(),
                                       dw.data_ptr(), B, T, C, KERNEL_WIDTH, 1, ws.data_ptr(), ws.numel(),
                                       N.stream_of(x)), "kdn_short_conv_bwd")
        return dx, dw, None


def qkv_causal_conv1d(x, weight):
    """SiLU causal convolution of packed q/k/v channels: (q, k, v)."""
    _validate_qkv_conv_inputs(x, weight)
    return _ShortConv.apply(x, weight, GROUPS)


def fixed_short_conv(convolution, hidden_states):
    """The diagonal mixer's per-tensor SiLU short convolution."""
    weight = convolution.weight
    if weight.ndim != 3 or weight.shape[1] != 1 or weight.shape[2] != KERNEL_WIDTH:
        raise ValueError(f"expected a depthwise [D, 1, {KERNEL_WIDTH}] convolution weight, got {tuple(weight.shape)}")
    if hidden_states.ndim != 3 or hidden_states.shape[-1] != weight.shape[0]:
        raise ValueError("hidden_states must be [B, T, D] with D the convolution's channels")
    w = weight.reshape(weight.shape[0], KERNEL_WIDTH)
    return _ShortConv.apply(hidden_states.contiguous(), w.contiguous() if not w.is_contiguous() else w, 1)[0]


__all__ = ("qkv_causal_conv1d", "fixed_short_conv")
