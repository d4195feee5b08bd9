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

import ctypes
from dataclasses import dataclass
from typing import Callable, Sequence

import torch
import torch.distributed as dist

from . import _native as N
from . import _scan
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


# ----------------------------------------------------------------------------- two-pass sequence parallelism
#
# The relay above makes rank r wait for rank r-1's whole segment.  The two
# passes below let every rank work at once.  Both carried states enter a
# segment through maps that do not depend on them:
#   covariance  p_end = M(p_in), a per-channel Moebius map (the composition of
#               the per-token maps p -> p_hat / (1 + u p_hat),
#               p_hat = alpha^2 p + omega, diag_kdn_naive.py:256-276);
#   memory      S_end = Phi S_in + S_end|0, Phi (K x K) the state reached from
#               the identity with zero values, S_end|0 the state reached from
#               zero (the recurrence is affine in S, diag_kdn_naive.py:479-500);
# and the adjoints leave it through the transposed maps:
#   dS_in = Phi^T dS_end + dS_in|0,   dp_in = A dp_end + dp_in|0 (per channel).
# Forward: every rank computes M and (Phi, S_end|0) of its segment, one
# all-gather shares them, each rank composes those of the ranks before it
# into its true incoming (p, S), then runs the covariance carry + emit and
# the sequential pass again from them.  Backward: every rank computes
# dS_in|0 (its reverse sweep from a zero final adjoint), one all-gather,
# each rank composes the ranks after it into its true final adjoint and runs
# the full backward; then the same for the covariance cotangent.  The
# chunk-parallel passes run once; only the sequential sweeps run twice (the
# state-map forward sweep carries two states in one launch).


class GroupComm:
    """All-gather over a torch.distributed group (NCCL for CUDA tensors, e.g.
    over NVLink on one box; gloo for CPU tensors)."""

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        t = t.contiguous()
        out = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        if t.is_cuda:
            dist.all_gather_into_tensor(out, t, group=self.group)
        else:
            dist.all_gather(list(out.unbind(0)), t, group=self.group)
        return out


def mobius_apply(m: torch.Tensor, p: torch.Tensor) -> torch.Tensor:
    """p -> (A p + B) / (C p + D) with m [..., 4] = (A, B, C, D)."""
    return (m[..., 0] * p + m[..., 1]) / (m[..., 2] * p + m[..., 3])


def carried_covariance(maps: torch.Tensor, p_first: torch.Tensor, rank: int) -> torch.Tensor:
    """Covariance entering segment ``rank``: the composed maps of the
    segments before it ([world, ...] stacked) applied to the first segment's
    incoming covariance."""
    p = p_first
    for j in range(rank):
        p = mobius_apply(maps[j], p)
    return p


def carried_state(phi: torch.Tensor, off: torch.Tensor, rank: int):
    """Memory state entering segment ``rank`` (None = zero, for rank 0):
    S_in(r) = Phi_{r-1} S_in(r-1) + off_{r-1} from S_in(0) = 0."""
    S = None
    for j in range(rank):
        S = off[j].clone() if S is None else torch.matmul(phi[j], S) + off[j]
    return S


def carried_state_adjoint(phi: torch.Tensor, c: torch.Tensor, rank: int):
    """Cotangent of segment ``rank``'s final state (None = zero, for the last
    rank): dS_end(r) = Phi_{r+1}^T dS_end(r+1) + c_{r+1}."""
    dS = None
    for j in range(phi.shape[0] - 1, rank, -1):
        dS = c[j].clone() if dS is None else torch.matmul(phi[j].transpose(-1, -2), dS) + c[j]
    return dS


def carried_covariance_adjoint(adj: torch.Tensor, rank: int):
    """Cotangent of segment ``rank``'s final covariance (None = zero, for the
    last rank) from the segments' composed adjoint maps adj [world, ..., 2]."""
    lam = None
    for j in range(adj.shape[0] - 1, rank, -1):
        lam = adj[j][..., 1].clone() if lam is None else adj[j][..., 0] * lam + adj[j][..., 1]
    return lam


class DiagSegmentB200:
    """One rank's segment of the diagonal KDN on the B200 kernels, pass by
    pass (the C ABI's split gain phases and partial scan modes).  Inputs are
    this rank's [B, T_r, H, D] slices, contiguous, as the operators take
    them; ``prior`` is the per-head initial precision."""

    def __init__(self, q, k, v, g_cumsum, k_gain, alpha, omega, r, prior, omega_raw, r_raw, scale):
        N.require_cuda(q, k, v, g_cumsum, k_gain, alpha, omega, r, prior, omega_raw, r_raw)
        self.t = dict(q=q, k=k, v=v, g=g_cumsum, k_gain=k_gain, alpha=alpha, omega=omega, r=r, prior=prior,
                      omega_raw=omega_raw, r_raw=r_raw)
        self.B, self.T, self.H, self.K = q.shape
        self.scale = float(scale)
        self.lib = N.load_library()
        self.dev = q.device
        self.stream = N.stream_of(q)
        self.gain_ws = N.byte_buffer(self.lib.kdn_diag_gain_workspace_bytes(self.B, self.T, self.H, self.K), self.dev)

    def _f32(self, *shape):
        return torch.empty(*shape, dtype=torch.float32, device=self.dev)

    def _gain_in(self):
        t = self.t
        return t["k_gain"].data_ptr(), t["alpha"].data_ptr(), t["omega"].data_ptr(), t["r"].data_ptr()

    def prior_covariance(self):
        return (1.0 / self.t["prior"]).view(1, self.H, 1).expand(self.B, self.H, self.K).contiguous()

    def S_end_template(self):
        return self._f32(self.B, self.H, self.K, self.t["v"].shape[-1])

    def cotangent(self, dO):
        """chunk_kalman's cotangent: fp32 at the boundary (the kernels round it to bf16)."""
        return dO.float().contiguous()

    # covariance, forward
    def gain_maps(self):
        total = self._f32(self.B, self.H, self.K, 4)
        N.check(self.lib.kdn_diag_gain_fwd_maps(*self._gain_in(), total.data_ptr(), self.B, self.T, self.H, self.K,
                                                self.gain_ws.data_ptr(), self.gain_ws.numel(), self.stream),
                "kdn_diag_gain_fwd_maps")
        return total

    def gain_finish(self, p_in):
        self.p_in = None if p_in is None else p_in.contiguous()
        self.kappa = self._f32(self.B, self.T, self.H, self.K)
        self.carry = self._f32(self.lib.kdn_diag_gain_carry_elems(self.B, self.T, self.H, self.K))
        N.check(self.lib.kdn_diag_gain_fwd_finish(*self._gain_in(), self.t["prior"].data_ptr(), N.ptr(self.p_in),
                                                  self.kappa.data_ptr(), self.carry.data_ptr(), None, self.B, self.T,
                                                  self.H, self.K, self.gain_ws.data_ptr(), self.gain_ws.numel(),
                                                  self.stream), "kdn_diag_gain_fwd_finish")

    # memory, forward
    def _args(self, mode):
        t = self.t
        a = _scan._args(N.KDN_DIAG, N.KDN_PREC_BF16, t["q"], t["v"], self.scale)
        a.mode = mode
        a.q, a.k, a.v, a.g = t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(), t["g"].data_ptr()
        a.kappa = self.kappa.data_ptr()
        return a

    def scan_summary(self):
        """(S_end|0, Phi) of the segment; leaves the chunk records in `saved`."""
        a = self._args(N.KDN_SCAN_FWD_RECORDS)
        self.saved = N.byte_buffer(self.lib.kdn_scan_saved_bytes(ctypes.byref(a)), self.dev)
        a.saved = self.saved.data_ptr()
        N.check(self.lib.kdn_scan_fwd(ctypes.byref(a), self.stream), "kdn_scan_fwd (records)")
        _scan.check_status(self.saved, "kdn_scan_fwd (records)")
        off, phi = self._f32(self.B, self.H, self.K, self.K), self._f32(self.B, self.H, self.K, self.K)
        a.mode = N.KDN_SCAN_FWD_STATE_MAP
        a.final_state, a.final_state_map = off.data_ptr(), phi.data_ptr()
        N.check(self.lib.kdn_scan_fwd(ctypes.byref(a), self.stream), "kdn_scan_fwd (state map)")
        _scan.check_status(self.saved, "kdn_scan_fwd (state map)")
        return off, phi

    def scan_sequential(self, S_in):
        a = self._args(N.KDN_SCAN_FWD_SEQUENTIAL)
        o = self._f32(self.B, self.T, self.H, self.K)
        self.S_in = None if S_in is None else S_in.contiguous()
        a.saved, a.o, a.initial_state = self.saved.data_ptr(), o.data_ptr(), N.ptr(self.S_in)
        N.check(self.lib.kdn_scan_fwd(ctypes.byref(a), self.stream), "kdn_scan_fwd (sequential)")
        _scan.check_status(self.saved, "kdn_scan_fwd (sequential)")
        return o

    # memory, backward
    def scan_adjoint_summary(self, dO):
        """dS_in with a zero final-state cotangent (the reverse sweep only)."""
        a = self._args(N.KDN_SCAN_BWD_STATE)
        ws = N.byte_buffer(self.lib.kdn_scan_workspace_bytes(ctypes.byref(a)), self.dev)
        c = self._f32(self.B, self.H, self.K, self.K)
        a.saved, a.dO, a.d_initial_state = self.saved.data_ptr(), dO.data_ptr(), c.data_ptr()
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        N.check(self.lib.kdn_scan_bwd(ctypes.byref(a), self.stream), "kdn_scan_bwd (state)")
        _scan.check_status(ws, "kdn_scan_bwd (state)")
        return c

    def scan_backward(self, dO, dS_end):
        t = self.t
        a = self._args(N.KDN_SCAN_FULL)
        ws = N.byte_buffer(self.lib.kdn_scan_workspace_bytes(ctypes.byref(a)), self.dev)
        dq, dk, dv = (torch.empty_like(t[n]) for n in ("q", "k", "v"))
        dg, dkappa = torch.empty_like(t["g"]), torch.empty_like(self.kappa)
        dS_end = None if dS_end is None else dS_end.contiguous()
        a.saved, a.dO, a.d_final_state = self.saved.data_ptr(), dO.data_ptr(), N.ptr(dS_end)
        a.dq, a.dk, a.dv, a.dg, a.dkappa = dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), dkappa.data_ptr()
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        N.check(self.lib.kdn_scan_bwd(ctypes.byref(a), self.stream), "kdn_scan_bwd")
        _scan.check_status(ws, "kdn_scan_bwd")
        self.dkappa = dkappa
        return dq, dk, dv, dg

    # covariance, backward
    def gain_adjoint_summary(self):
        total = self._f32(self.B, self.H, self.K, 2)
        self.gain_bws = N.byte_buffer(self.lib.kdn_diag_gain_workspace_bytes(self.B, self.T, self.H, self.K), self.dev)
        N.check(self.lib.kdn_diag_gain_bwd_maps(*self._gain_in(), self.dkappa.data_ptr(), self.carry.data_ptr(),
                                                total.data_ptr(), self.B, self.T, self.H, self.K,
                                                self.gain_bws.data_ptr(), self.gain_bws.numel(), self.stream),
                "kdn_diag_gain_bwd_maps")
        return total

    def gain_backward(self, lam_end):
        t = self.t
        dk_gain, dalpha = torch.empty_like(t["k_gain"]), torch.empty_like(t["alpha"])
        domega_raw, dr_raw = torch.empty_like(t["omega_raw"]), torch.empty_like(t["r_raw"])
        dprior = self._f32(self.H)
        lam_end = None if lam_end is None else lam_end.contiguous()
        N.check(self.lib.kdn_diag_gain_bwd_finish(
            *self._gain_in(), t["prior"].data_ptr(), N.ptr(self.p_in), t["omega_raw"].data_ptr(),
            t["r_raw"].data_ptr(), self.dkappa.data_ptr(), self.carry.data_ptr(), N.ptr(lam_end),
            dk_gain.data_ptr(), dalpha.data_ptr(), domega_raw.data_ptr(), dr_raw.data_ptr(), dprior.data_ptr(), None,
            self.B, self.T, self.H, self.K, self.gain_bws.data_ptr(), self.gain_bws.numel(), self.stream),
            "kdn_diag_gain_bwd_finish")
        if self.p_in is not None:  # the prior reaches this segment only through the carried covariance
            dprior.zero_()
        return dk_gain, dalpha, domega_raw, dr_raw, dprior


class IsoSegmentB200:
    """One rank's segment of the isotropic KDN on the B200 kernels, pass by
    pass (the C ABI's split gain phases and partial scan modes); the same
    interface as DiagSegmentB200 with a scalar covariance per (b, h).  Inputs
    are this rank's [B, T_r, H, *] slices (q, k, v bf16; g_cumsum fp32
    64-local; a, omega, r fp32 [B, T_r, H]); ``prior`` is the per-head initial
    precision."""

    def __init__(self, q, k, v, g_cumsum, a, omega, r, prior, scale, posterior_scale=1.0):
        N.require_cuda(q, k, v, g_cumsum, a, omega, r, prior)
        self.t = dict(q=q, k=k, v=v, g=g_cumsum, a=a, omega=omega, r=r, prior=prior)
        self.B, self.T, self.H, self.K = q.shape
        self.scale, self.s = float(scale), float(posterior_scale)
        self.lib = N.load_library()
        self.dev = q.device
        self.stream = N.stream_of(q)
        self.gain_ws = N.byte_buffer(self.lib.kdn_iso_gain_workspace_bytes(self.B, self.T, self.H), self.dev)

    def _f32(self, *shape):
        return torch.empty(*shape, dtype=torch.float32, device=self.dev)

    def _gain_in(self):
        t = self.t
        return t["a"].data_ptr(), t["omega"].data_ptr(), t["r"].data_ptr()

    def prior_covariance(self):
        return (1.0 / self.t["prior"]).view(1, self.H).expand(self.B, self.H).contiguous()

    def S_end_template(self):
        return self._f32(self.B, self.H, self.K, self.t["v"].shape[-1])

    def cotangent(self, dO):
        """The isotropic scan's cotangent is bf16, like its output."""
        return dO.to(torch.bfloat16).contiguous()

    # covariance, forward
    def gain_maps(self):
        total = self._f32(self.B, self.H, 4)
        N.check(self.lib.kdn_iso_gain_fwd_maps(*self._gain_in(), total.data_ptr(), self.B, self.T, self.H, self.s,
                                               self.gain_ws.data_ptr(), self.gain_ws.numel(), self.stream),
                "kdn_iso_gain_fwd_maps")
        return total

    def gain_finish(self, p_in):
        self.p_in = None if p_in is None else p_in.contiguous()
        self.beta = self._f32(self.B, self.T, self.H)
        self.p_prev = self._f32(self.B, self.T, self.H)
        N.check(self.lib.kdn_iso_gain_fwd_finish(*self._gain_in(), self.t["prior"].data_ptr(), N.ptr(self.p_in),
                                                 self.beta.data_ptr(), self.p_prev.data_ptr(), None, self.B, self.T,
                                                 self.H, self.s, self.gain_ws.data_ptr(), self.gain_ws.numel(),
                                                 self.stream), "kdn_iso_gain_fwd_finish")

    # memory, forward
    def _args(self, mode):
        t = self.t
        a = _scan._args(N.KDN_ISO, N.KDN_PREC_BF16, t["q"], t["v"], self.scale)
        a.mode = mode
        a.q, a.k, a.v, a.g = t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(), t["g"].data_ptr()
        a.beta = self.beta.data_ptr()
        return a

    def scan_summary(self):
        return DiagSegmentB200.scan_summary(self)

    def scan_sequential(self, S_in):
        a = self._args(N.KDN_SCAN_FWD_SEQUENTIAL)
        o = torch.empty(self.B, self.T, self.H, self.t["v"].shape[-1], dtype=torch.bfloat16, device=self.dev)
        self.S_in = None if S_in is None else S_in.contiguous()
        a.saved, a.o, a.initial_state = self.saved.data_ptr(), o.data_ptr(), N.ptr(self.S_in)
        N.check(self.lib.kdn_scan_fwd(ctypes.byref(a), self.stream), "kdn_scan_fwd (sequential)")
        _scan.check_status(self.saved, "kdn_scan_fwd (sequential)")
        return o

    # memory, backward
    def scan_adjoint_summary(self, dO):
        return DiagSegmentB200.scan_adjoint_summary(self, dO)

    def scan_backward(self, dO, dS_end):
        t = self.t
        a = self._args(N.KDN_SCAN_FULL)
        ws = N.byte_buffer(self.lib.kdn_scan_workspace_bytes(ctypes.byref(a)), self.dev)
        dq, dk, dv = (torch.empty_like(t[n]) for n in ("q", "k", "v"))
        dg, dbeta = torch.empty_like(t["g"]), torch.empty_like(self.beta)
        dS_end = None if dS_end is None else dS_end.contiguous()
        a.saved, a.dO, a.d_final_state = self.saved.data_ptr(), dO.data_ptr(), N.ptr(dS_end)
        a.dq, a.dk, a.dv, a.dg, a.dbeta = dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), dbeta.data_ptr()
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        N.check(self.lib.kdn_scan_bwd(ctypes.byref(a), self.stream), "kdn_scan_bwd")
        _scan.check_status(ws, "kdn_scan_bwd")
        self.dbeta = dbeta
        return dq, dk, dv, dg

    # covariance, backward
    def gain_adjoint_summary(self):
        total = self._f32(self.B, self.H, 2)
        self.gain_bws = N.byte_buffer(self.lib.kdn_iso_gain_workspace_bytes(self.B, self.T, self.H), self.dev)
        N.check(self.lib.kdn_iso_gain_bwd_maps(*self._gain_in(), self.dbeta.data_ptr(), self.p_prev.data_ptr(),
                                               total.data_ptr(), self.B, self.T, self.H, self.s,
                                               self.gain_bws.data_ptr(), self.gain_bws.numel(), self.stream),
                "kdn_iso_gain_bwd_maps")
        return total

    def gain_backward(self, lam_end):
        t = self.t
        da, domega, dr = (torch.empty_like(t[n]) for n in ("a", "omega", "r"))
        dprior = self._f32(self.H)
        lam_end = None if lam_end is None else lam_end.contiguous()
        N.check(self.lib.kdn_iso_gain_bwd_finish(
            *self._gain_in(), t["prior"].data_ptr(), N.ptr(self.p_in), self.dbeta.data_ptr(), self.p_prev.data_ptr(),
            N.ptr(lam_end), da.data_ptr(), domega.data_ptr(), dr.data_ptr(), dprior.data_ptr(), None, self.B, self.T,
            self.H, self.s, self.gain_bws.data_ptr(), self.gain_bws.numel(), self.stream), "kdn_iso_gain_bwd_finish")
        if self.p_in is not None:  # the prior reaches this segment only through the carried covariance
            dprior.zero_()
        return da, domega, dr, dprior


def two_pass_forward(seg, comm):
    """Forward of one rank's segment (diagonal or isotropic segment object):
    returns o and the gathered state maps the backward needs."""
    rank = comm.rank
    maps = comm.all_gather(seg.gain_maps())
    seg.gain_finish(None if rank == 0 else carried_covariance(maps, seg.prior_covariance(), rank))
    off, phi = seg.scan_summary()
    if phi.shape == off.shape:  # K = V: one all-gather, [world, 2, B, H, K, K]
        both = comm.all_gather(torch.stack((phi, off)))
        phis, offs = both[:, 0], both[:, 1]
    else:
        phis, offs = comm.all_gather(phi), comm.all_gather(off)
    o = seg.scan_sequential(carried_state(phis, offs, rank))
    return o, phis


def two_pass_backward(seg, comm, phis, dO):
    """Backward of one rank's segment: returns (dq, dk, dv, dg) followed by
    the segment's gain gradients (diagonal: dk_gain, dalpha, domega_raw,
    dr_raw, dprior; isotropic: da, domega, dr, dprior); dprior is nonzero on
    rank 0 only (sum it over ranks like any parameter gradient)."""
    rank = comm.rank
    dO = seg.cotangent(dO)
    # rank 0's own summaries are needed by no one: it sends zeros of their shapes
    c = seg.scan_adjoint_summary(dO) if rank > 0 else torch.zeros_like(seg.S_end_template())
    cs = comm.all_gather(c)
    dq, dk, dv, dg = seg.scan_backward(dO, carried_state_adjoint(phis, cs, rank))
    adj = seg.gain_adjoint_summary()  # rank 0 needs its segment maps for the finish all the same
    adjs = comm.all_gather(adj if rank > 0 else torch.zeros_like(adj))
    return (dq, dk, dv, dg) + tuple(seg.gain_backward(carried_covariance_adjoint(adjs, rank)))


# the diagonal names of the drivers
diag_two_pass_forward = two_pass_forward
diag_two_pass_backward = two_pass_backward


class _DiagTwoPass(torch.autograd.Function):
    @staticmethod
    def forward(ctx, comm, scale, q, k, v, g_cumsum, k_gain, alpha, omega, r, prior, omega_raw, r_raw):
        seg = DiagSegmentB200(q, k, v, g_cumsum, k_gain, alpha, omega, r, prior, omega_raw, r_raw, scale)
        o, phis = diag_two_pass_forward(seg, comm)
        ctx.state = (seg, comm, phis)
        return o

    @staticmethod
    def backward(ctx, do):
        seg, comm, phis = ctx.state
        if do is None:
            do = torch.zeros(seg.B, seg.T, seg.H, seg.K, dtype=torch.float32, device=seg.dev)
        grads = diag_two_pass_backward(seg, comm, phis, do)
        del ctx.state
        dq, dk, dv, dg, dk_gain, dalpha, domega_raw, dr_raw, dprior = grads
        return None, None, dq, dk, dv, dg, dk_gain, dalpha, None, None, dprior, domega_raw, dr_raw


def sp_diag_kdn_two_pass(q, k, v, g_cumsum, k_gain, alpha, omega, r, initial_precision, omega_raw, r_raw, *,
                         group=None, comm=None, scale=None):
    """This rank's output of the sequence-parallel diagonal KDN (gain +
    memory scan), every rank working at once (see the two-pass notes above).
    Inputs are this rank's contiguous time slice, a multiple of 32 tokens
    except on the last rank; bf16 precision only.  ``initial_precision``
    receives its gradient on rank 0 (sum parameter gradients over ranks)."""
    comm = GroupComm(group) if comm is None else comm
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    if N.precision() != N.KDN_PREC_BF16:
        raise ValueError("the two-pass sequence-parallel scan runs the bf16 tensor-core kernels only")
    cont = [t.contiguous() for t in (q, k, v, g_cumsum, k_gain, alpha, omega.detach(), r.detach(),
                                      initial_precision, omega_raw, r_raw)]
    return _DiagTwoPass.apply(comm, scale, *cont)


class _IsoTwoPass(torch.autograd.Function):
    @staticmethod
    def forward(ctx, comm, scale, posterior_scale, q, k, v, g_cumsum, a, omega, r, prior):
        seg = IsoSegmentB200(q, k, v, g_cumsum, a, omega, r, prior, scale, posterior_scale)
        o, phis = two_pass_forward(seg, comm)
        ctx.state = (seg, comm, phis)
        return o

    @staticmethod
    def backward(ctx, do):
        seg, comm, phis = ctx.state
        if do is None:
            do = torch.zeros(seg.B, seg.T, seg.H, seg.K, dtype=torch.bfloat16, device=seg.dev)
        dq, dk, dv, dg, da, domega, dr, dprior = two_pass_backward(seg, comm, phis, do)
        del ctx.state
        return None, None, None, dq, dk, dv, dg, da, domega, dr, dprior


def sp_iso_kdn_two_pass(q, k, v, g_cumsum, a, omega, r, initial_precision, *, group=None, comm=None, head_dim=128,
                        info_scale=None, scale=None):
    """This rank's output (bf16) of the sequence-parallel isotropic KDN
    (``iso_kdn_gain`` + ``_chunk_kda_precumsum_paired``), every rank working
    at once (the two passes above with a scalar covariance per (b, h)).
    Inputs are this rank's contiguous time slice, a multiple of 64 tokens
    except on the last rank; q, k, v bf16 with K = V = 128; bf16 precision
    only.  ``initial_precision`` receives its gradient on rank 0 (sum
    parameter gradients over ranks)."""
    comm = GroupComm(group) if comm is None else comm
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    posterior_scale = (float(head_dim) if info_scale is None else float(info_scale)) / float(head_dim)
    if N.precision() != N.KDN_PREC_BF16:
        raise ValueError("the two-pass sequence-parallel scan runs the bf16 tensor-core kernels only")
    cont = [t.contiguous() for t in (q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16), g_cumsum,
                                      a.float(), omega.float(), r.float(), initial_precision.float())]
    return _IsoTwoPass.apply(comm, scale, posterior_scale, *cont)
