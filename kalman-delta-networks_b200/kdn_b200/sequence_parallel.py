"""Sequence parallelism for the KDN scan: one long sequence split over ranks.

The time axis is split contiguously over the ranks of a process group.  Rank r
runs its segment from the memory state S (fp32 [B,H,K,V]) and covariance p
(iso fp32 [B,H], diag fp32 [B,H,K]) that rank r-1 ended with and hands its own
final (S, p) to rank r+1 with NCCL point-to-point send/recv (over NVLink on one
box).  The backward runs the chain in reverse with the cotangents (dS, dp).
Rank 0 starts from S = 0 and p = 1/initial_precision; only rank 0's
``initial_precision`` therefore receives a gradient from the covariance path.

Segment boundaries must fall on gate-chunk boundaries (multiples of 64 tokens
for the isotropic scan, 32 for the diagonal scan) so that each rank's
``g_cumsum`` is the same chunk-local prefix the full sequence would have.

The reference has no sequence parallelism (its mixers reject caches and
states, iso_kdn.py:228-240); the state recurrences continued here are the ones
of iso_kdn_naive.py:238-251 / diag_kdn_naive.py:256-276 (covariance) and
the memory recurrence, with ``initial_memory`` / ``initial_precision``
(iso_kdn_naive.py:376-388).

``chain(segment_fn, inputs, link)`` is independent of where the segment runs:
``iso_segment`` / ``diag_segment`` below run it on the B200 kernels; the
tests run it on CPU ranks (gloo) with the oracle as ``segment_fn``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import torch
import torch.distributed as dist

from . import _native as N
from ._scan import ScanSaved, scan_backward, scan_forward


# ----------------------------------------------------------------------------- links


@dataclass
class Link:
    """Neighbours of this rank in the chain (global ranks, None at the ends)."""

    prev: int | None
    next: int | None
    group: object = None

    @staticmethod
    def from_group(group=None) -> "Link":
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        to_global = (lambda r: dist.get_global_rank(group, r)) if group is not None else (lambda r: r)
        return Link(
            prev=to_global(rank - 1) if rank > 0 else None,
            next=to_global(rank + 1) if rank + 1 < world else None,
            group=group,
        )

    def send(self, tensors: Sequence[torch.Tensor], dst: int) -> None:
        for t in tensors:
            dist.send(t.contiguous(), dst, group=self.group)

    def recv(self, templates: Sequence[torch.Tensor], src: int) -> list[torch.Tensor]:
        out = []
        for t in templates:
            buf = torch.empty_like(t)
            dist.recv(buf, src, group=self.group)
            out.append(buf)
        return out


class _Chain(torch.autograd.Function):
    """Run ``fn(*inputs, *states_in) -> (out, *states_out)`` between a receive
    from the previous rank and a send to the next; reverse in backward."""

    @staticmethod
    def forward(ctx, fn, link, state_templates, n_inputs, *inputs):
        states_in = None if link.prev is None else link.recv(state_templates, link.prev)
        with torch.enable_grad():
            xs = [x.detach().requires_grad_(x.requires_grad) if isinstance(x, torch.Tensor) else x for x in inputs]
            ss = None if states_in is None else [s.requires_grad_(True) for s in states_in]
            out, *finals = fn(*xs, *(ss if ss is not None else [None] * len(state_templates)))
        if link.next is not None:
            link.send([f.detach() for f in finals], link.next)
        ctx.fn_graph = (xs, ss, out, finals)
        ctx.link = link
        return out.detach()

    @staticmethod
    def backward(ctx, dout):
        xs, ss, out, finals = ctx.fn_graph
        link = ctx.link
        d_finals = (
            [torch.zeros_like(f) for f in finals] if link.next is None else link.recv([f.detach() for f in finals], link.next)
        )
        wrt = [x for x in xs if isinstance(x, torch.Tensor) and x.requires_grad] + (ss or [])
        grads = torch.autograd.grad([out, *finals], wrt, [dout, *d_finals], allow_unused=True)
        n_x = len(wrt) - len(ss or [])
        if link.prev is not None:
            link.send([g if g is not None else torch.zeros_like(s) for g, s in zip(grads[n_x:], ss)], link.prev)
        it = iter(grads[:n_x])
        dx = [next(it) if isinstance(x, torch.Tensor) and x.requires_grad else None for x in xs]
        del ctx.fn_graph
        return (None, None, None, None, *dx)


def chain(segment_fn: Callable, inputs: Sequence, state_templates: Sequence[torch.Tensor], link: Link) -> torch.Tensor:
    """Differentiable sequence-parallel run of ``segment_fn`` on this rank's
    segment.  ``state_templates`` give the shapes/dtypes/devices of the carried
    states; ``segment_fn`` receives ``None`` for them on the first rank."""
    return _Chain.apply(segment_fn, link, list(state_templates), len(inputs), *inputs)


# ----------------------------------------------------------------------------- B200 segment ops


class _IsoGainSegment(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, omega, r, initial_precision, p0, posterior_scale):
        from .iso_kdn_chunk import _iso_gain_forward

        beta, p_prev, p_final = _iso_gain_forward(
            a, omega, r, initial_precision, out_dtype=torch.float32, save_state=True,
            posterior_scale=posterior_scale, initial_cov=p0, want_final=True,
        )
        ctx.save_for_backward(a, omega, r, initial_precision, p_prev, p0)
        ctx.has_p0 = p0 is not None
        ctx.posterior_scale = posterior_scale
        return beta, p_final

    @staticmethod
    def backward(ctx, dbeta, dp_final):
        from .iso_kdn_chunk import _iso_gain_backward

        a, omega, r, initial_precision, p_prev, p0 = ctx.saved_tensors
        dbeta = torch.zeros_like(a) if dbeta is None else dbeta
        da, domega, dr, dinit, dp0 = _iso_gain_backward(
            a, omega, r, initial_precision, dbeta, p_prev, posterior_scale=ctx.posterior_scale,
            initial_cov=p0 if ctx.has_p0 else None, d_final_cov=dp_final, want_d_initial=ctx.has_p0,
        )
        return da, domega, dr, dinit, dp0, None


class _ScanSegment(torch.autograd.Function):
    @staticmethod
    def forward(ctx, variant, q, k, v, g, gate, S0, scale):
        in_dtype = q.dtype
        if variant == N.KDN_ISO:
            q, k, v = (x.to(torch.bfloat16).contiguous() for x in (q, k, v))
            gate = gate.float().contiguous()
        o, S_T, saved = scan_forward(variant, q, k, v, g.contiguous(), gate, scale, initial_state=S0,
                                     want_final_state=True)
        ctx.save_for_backward(q, k, v, g, gate, saved.saved)
        ctx.meta = (variant, saved.precision, scale, S0 is not None, in_dtype)
        return (o.to(in_dtype) if variant == N.KDN_ISO else o), S_T

    @staticmethod
    def backward(ctx, do, dS_T):
        q, k, v, g, gate, saved = ctx.saved_tensors
        variant, precision, scale, has_S0, in_dtype = ctx.meta
        if do is None:
            do = torch.zeros(v.shape, dtype=torch.float32, device=v.device)
        dO = do.to(torch.bfloat16 if variant == N.KDN_ISO else torch.float32).contiguous()
        dq, dk, dv, dg, dgate, dS0 = scan_backward(
            variant, q, k, v, g, gate, scale, ScanSaved(saved, precision), dO,
            d_final_state=None if dS_T is None else dS_T.contiguous(), want_d_initial=has_S0,
        )
        return None, dq.to(in_dtype), dk.to(in_dtype), dv.to(in_dtype), dg, dgate, dS0, None


class _DiagGainSegment(torch.autograd.Function):
    @staticmethod
    def forward(ctx, k, alpha, omega, r, initial_precision, omega_raw, r_raw, p0):
        from .diag_kdn_chunk import _gain_forward

        kappa, carry, p_final = _gain_forward(k, alpha, omega, r, initial_precision, initial_cov=p0, want_final=True)
        ctx.save_for_backward(k, alpha, omega, r, initial_precision, omega_raw, r_raw, carry, p0)
        ctx.has_p0 = p0 is not None
        return kappa, p_final

    @staticmethod
    def backward(ctx, dkappa, dp_final):
        from .diag_kdn_chunk import _gain_backward

        k, alpha, omega, r, initial_precision, omega_raw, r_raw, carry, p0 = ctx.saved_tensors
        dk, dalpha, domega_raw, dr_raw, dinit, dp0 = _gain_backward(
            k, alpha, omega, r, initial_precision, omega_raw, r_raw, dkappa, carry, need_initial=True,
            initial_cov=p0 if ctx.has_p0 else None, d_final_cov=dp_final, want_d_initial=ctx.has_p0,
        )
        return dk, dalpha, None, None, dinit, domega_raw, dr_raw, dp0


def iso_segment(q, k, v, g_cumsum, a, omega, r, initial_precision, S0=None, p0=None, *, head_dim=128,
                info_scale=None, scale=None):
    """Isotropic gain + memory scan of one segment with carried-in state.
    Returns ``(o, S_T, p_T)``, differentiable in every tensor argument."""
    posterior_scale = (float(head_dim) if info_scale is None else float(info_scale)) / float(head_dim)
    beta, p_T = _IsoGainSegment.apply(a.contiguous(), omega.contiguous(), r.contiguous(),
                                      initial_precision.contiguous(), p0, posterior_scale)
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    o, S_T = _ScanSegment.apply(N.KDN_ISO, q, k, v, g_cumsum, beta, S0, scale)
    return o, S_T, p_T


def diag_segment(q, k, v, g_cumsum, k_gain, alpha, omega, r, initial_precision, omega_raw, r_raw, S0=None, p0=None,
                 *, scale=None):
    """Diagonal gain + memory scan of one segment with carried-in state.
    Returns ``(o fp32, S_T, p_T)``."""
    kappa, p_T = _DiagGainSegment.apply(k_gain, alpha, omega.detach(), r.detach(), initial_precision, omega_raw,
                                        r_raw, p0)
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    o, S_T = _ScanSegment.apply(N.KDN_DIAG, q, k, v, g_cumsum, kappa, S0, scale)
    return o, S_T, p_T


def sp_iso_kdn(q, k, v, g_cumsum, a, omega, r, initial_precision, *, group=None, head_dim=128, info_scale=None):
    """This rank's output of the sequence-parallel isotropic KDN scan."""
    B, T, H, K = q.shape
    templates = [torch.empty(B, H, K, v.shape[-1], device=q.device), torch.empty(B, H, device=q.device)]

    def fn(q, k, v, g, a, omega, r, prec, S0, p0):
        return iso_segment(q, k, v, g, a, omega, r, prec, S0, p0, head_dim=head_dim, info_scale=info_scale)

    return chain(fn, (q, k, v, g_cumsum, a, omega, r, initial_precision), templates, Link.from_group(group))


def sp_diag_kdn(q, k, v, g_cumsum, k_gain, alpha, omega, r, initial_precision, omega_raw, r_raw, *, group=None):
    """This rank's output of the sequence-parallel diagonal KDN scan."""
    B, T, H, K = q.shape
    templates = [torch.empty(B, H, K, v.shape[-1], device=q.device), torch.empty(B, H, K, device=q.device)]

    def fn(q, k, v, g, kg, alpha, omega, r, prec, wr, rr, S0, p0):
        return diag_segment(q, k, v, g, kg, alpha, omega, r, prec, wr, rr, S0, p0)

    return chain(fn, (q, k, v, g_cumsum, k_gain, alpha, omega, r, initial_precision, omega_raw, r_raw), templates,
                 Link.from_group(group))
