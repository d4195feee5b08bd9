"""TEST INFRASTRUCTURE ONLY -- tokenwise CPU restatement of the KDN recurrences.

Every function here is a plain PyTorch loop over tokens, evaluated in float64
by default, and exists only to check the CUDA operators.  Citations are to the
reference tree (``lit_gpt/kdn_ops/...``) the restatement follows.

Conventions shared with the operators under test
------------------------------------------------
* ``g_cumsum`` is the base-2 inclusive prefix of ``ln(alpha)`` that restarts
  every ``chunk`` tokens (64 for the isotropic scan, 32 for the diagonal scan):
  ``g_cumsum[t] = log2(e) * sum_{s in chunk(t), s <= t} ln(alpha[s])``
  (producer: iso_kdn_chunk.py:787-792, diag_kdn_chunk.py:1889-1898).
* The scan's gradient for ``g_cumsum`` is returned in natural-log coordinates
  and before the reverse chunk cumsum (iso_kdn_chunk.py:2180-2186,
  933-936; diag_kdn_chunk.py:1990-1996).  With ``G = ln(2) * g_cumsum`` that is
  exactly ``dL/dG`` evaluated position by position, which is what
  :func:`scan_grads` returns.
"""
from __future__ import annotations

import math

import torch

__all__ = (
    "LN2",
    "l2norm",
    "alpha_from_g_cumsum",
    "g_cumsum_from_log_alpha",
    "iso_gain",
    "diag_gain",
    "memory_recurrence",
    "iso_scan",
    "diag_scan",
    "iso_gain_grads",
    "diag_gain_grads",
    "scan_grads",
    "make_iso_inputs",
    "make_diag_inputs",
    "iso_gate",
    "iso_gate_grads",
    "make_iso_gate_inputs",
    "DIAG_ALPHA_FLOOR",
    "diag_gate",
    "diag_gate_grads",
    "make_diag_gate_inputs",
    "diag_normalize",
    "diag_normalize_backward",
    "rms_norm_gated",
    "short_conv",
)

LN2 = math.log(2.0)
L2NORM_EPS = 1e-6


def l2norm(x: torch.Tensor, eps: float = L2NORM_EPS) -> torch.Tensor:
    """x / sqrt(sum(x^2) + eps) over the last axis (FLA ``l2norm_fwd``, the
    normalisation ``_ChunkKDAPrecumsumFunction`` applies, iso_kdn_chunk.py:2203)."""
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def g_cumsum_from_log_alpha(log_alpha: torch.Tensor, chunk: int) -> torch.Tensor:
    """Chunk-local base-2 prefix of ``ln(alpha)`` along T (axis 1), the tensor the
    gate frontends hand to the scan (iso_kdn_chunk.py:787-792)."""
    B, T = log_alpha.shape[:2]
    out = torch.empty_like(log_alpha)
    for start in range(0, T, chunk):
        stop = min(start + chunk, T)
        out[:, start:stop] = log_alpha[:, start:stop].cumsum(1) / LN2
    return out


def alpha_from_g_cumsum(G: torch.Tensor, chunk: int) -> torch.Tensor:
    """Retention alpha from the NATURAL-log chunk-local prefix ``G = ln2 * g_cumsum``.

    ``ln(alpha[t]) = G[t] - G[t-1]`` inside a chunk and ``G[t]`` at a chunk's
    first token.  Differentiable in ``G``.
    """
    T = G.shape[1]
    prev = torch.zeros_like(G)
    prev[:, 1:] = G[:, :-1]
    starts = torch.arange(T, device=G.device) % chunk == 0
    shape = [1, T] + [1] * (G.ndim - 2)
    prev = torch.where(starts.view(shape), torch.zeros_like(G), prev)
    return torch.exp(G - prev)


def iso_gain(
    a: torch.Tensor,
    omega: torch.Tensor,
    r: torch.Tensor,
    initial_precision: torch.Tensor,
    posterior_scale: float = 1.0,
    initial_covariance: torch.Tensor | None = None,
):
    """Scalar covariance scan of ``iso_kdn_gain`` for unit-norm keys.

    Follows iso_kdn_naive.py:238-251 with ``||k||^2 = 1`` and the production
    parameterisation of iso_kdn_chunk.py:1552-1598 (``a = mean(alpha^2)`` given,
    ``posterior_scale = info_scale / head_dim``)::

        z_t = a_t * p_{t-1} + omega_t
        beta_t = z_t / (r_t + z_t)
        p_t = r_t * z_t / (r_t + posterior_scale * z_t)

    with ``p_{-1} = 1 / initial_precision[h]`` (or ``initial_covariance[b,h]``).
    Inputs are [B,T,H]; returns ``(beta [B,T,H], p_prev [B,T,H], p_final [B,H])``.
    """
    B, T, H = a.shape
    if initial_covariance is None:
        p = (1.0 / initial_precision).view(1, H).expand(B, H)
    else:
        p = initial_covariance
    betas, prevs = [], []
    for t in range(T):
        prevs.append(p)
        z = a[:, t] * p + omega[:, t]
        betas.append(z / (r[:, t] + z))
        p = r[:, t] * z / (r[:, t] + posterior_scale * z)
    if T == 0:
        empty = a.new_zeros((B, 0, H))
        return empty, empty, p
    return torch.stack(betas, 1), torch.stack(prevs, 1), p


def diag_gain(
    k: torch.Tensor,
    alpha: torch.Tensor,
    omega: torch.Tensor,
    r: torch.Tensor,
    initial_precision: torch.Tensor,
    info_scale: float | None = None,
    initial_covariance: torch.Tensor | None = None,
):
    """Per-channel covariance scan of ``_diag_kdn_gain`` (diag_kdn_naive.py:256-276)::

        p_hat_t = alpha_t^2 * p_{t-1} + omega_t
        kappa_t = p_hat_t * k_t / (r_t + sum_c p_hat_tc * k_tc^2)
        p_t     = p_hat_t / (1 + info_scale * k_t^2 / r_t * p_hat_t)

    ``info_scale`` defaults to K (the production value, diag_kdn_chunk.py:2525).
    k, alpha, omega are [B,T,H,K]; r is [B,T,H]; ``initial_precision`` is [H].
    Returns ``(kappa [B,T,H,K], p_final [B,H,K])``.
    """
    B, T, H, K = k.shape
    s = float(K) if info_scale is None else float(info_scale)
    if initial_covariance is None:
        p = (1.0 / initial_precision).view(1, H, 1).expand(B, H, K)
    else:
        p = initial_covariance
    gains = []
    for t in range(T):
        p_hat = alpha[:, t] ** 2 * p + omega[:, t]
        ksq = k[:, t] ** 2
        denom = r[:, t, :, None] + (p_hat * ksq).sum(-1, keepdim=True)
        gains.append(p_hat * k[:, t] / denom)
        u = s * ksq / r[:, t, :, None]
        p = p_hat / (1.0 + u * p_hat)
    if T == 0:
        return k.new_zeros((B, 0, H, K)), p
    return torch.stack(gains, 1), p


def memory_recurrence(q, k, v, alpha, kappa, S0, scale):
    """Tokenwise memory and readout (iso_kdn_naive.py:308-332,
    diag_kdn_naive.py:479-500)::

        S_hat = Diag(alpha_t) S;  delta = v_t - k_t^T S_hat
        S = S_hat + kappa_t delta^T;  o_t = scale * q_t^T S

    ``kappa`` is the write vector: ``beta_t * k_t`` for the isotropic scan, the
    diagonal gain for the diagonal scan.  q, k, alpha, kappa [B,T,H,K];
    v [B,T,H,V]; S0 [B,H,K,V].  Returns ``(o [B,T,H,V], S [B,H,K,V])``.
    """
    S = S0
    outs = []
    for t in range(q.shape[1]):
        S_hat = alpha[:, t, ..., None] * S
        delta = v[:, t] - torch.einsum("bhk,bhkv->bhv", k[:, t], S_hat)
        S = S_hat + kappa[:, t, ..., None] * delta[..., None, :]
        outs.append(scale * torch.einsum("bhk,bhkv->bhv", q[:, t], S))
    if not outs:
        return v.new_zeros(v.shape), S
    return torch.stack(outs, 1), S


def _scan(q_mem, k_mem, v, G, kappa, scale, chunk, S0):
    B, T, H, K = q_mem.shape
    V = v.shape[-1]
    if S0 is None:
        S0 = q_mem.new_zeros((B, H, K, V))
    alpha = alpha_from_g_cumsum(G, chunk)
    return memory_recurrence(q_mem, k_mem, v, alpha, kappa, S0, scale)


def iso_scan(q, k, v, g_cumsum, beta, scale=None, S0=None, dtype=torch.float64):
    """Forward of ``_chunk_kda_precumsum_paired`` (iso_kdn_chunk.py:2190-2212).

    q and k are L2-normalised inside the op, ``kappa_t = beta_t * k_hat_t`` and
    ``alpha`` comes from the 64-local base-2 ``g_cumsum``.  Returns ``(o, S_T)``
    in ``dtype``.
    """
    K = q.shape[-1]
    scale = K ** -0.5 if scale is None else scale
    qh = l2norm(q.to(dtype))
    kh = l2norm(k.to(dtype))
    G = g_cumsum.to(dtype) * LN2
    kappa = beta.to(dtype)[..., None] * kh
    S0 = None if S0 is None else S0.to(dtype)
    return _scan(qh, kh, v.to(dtype), G, kappa, scale, 64, S0)


def diag_scan(q, k, kappa, v, g_cumsum, scale, S0=None, dtype=torch.float64):
    """Forward of ``chunk_kalman`` (diag_kdn_chunk.py:3247-3332): memory keys and
    queries used as given, the gain ``kappa`` as the write vector and ``alpha``
    from the 32-local base-2 ``g_cumsum``.  Returns ``(o, S_T)`` in ``dtype``."""
    G = g_cumsum.to(dtype) * LN2
    S0 = None if S0 is None else S0.to(dtype)
    return _scan(q.to(dtype), k.to(dtype), v.to(dtype), G, kappa.to(dtype), scale, 32, S0)


def scan_grads(variant, inputs, dO, scale=None, S0=None, dS_T=None, dtype=torch.float64):
    """Autograd gradients of the scan op in the operator's own conventions.

    ``variant`` is "iso" (inputs q, k, v, g_cumsum, beta) or "diag" (inputs q, k,
    kappa, v, g_cumsum).  Returns a dict with ``o``, ``S_T`` and the gradients
    ``dq, dk, dv, dg`` plus ``dbeta`` (iso) or ``dkappa`` (diag), and ``dS0``
    when ``S0`` is given.  ``dg`` is the natural-log, pre-reverse cotangent.
    """
    leaves = {name: t.detach().to(dtype).clone().requires_grad_(True) for name, t in inputs.items()}
    G = (leaves["g_cumsum"] * LN2).detach().requires_grad_(True)
    S0_leaf = None if S0 is None else S0.detach().to(dtype).clone().requires_grad_(True)
    K = leaves["q"].shape[-1]
    if variant == "iso":
        sc = K ** -0.5 if scale is None else scale
        qh = l2norm(leaves["q"])
        kh = l2norm(leaves["k"])
        kappa = leaves["beta"][..., None] * kh
        o, S = _scan(qh, kh, leaves["v"], G, kappa, sc, 64, S0_leaf)
    else:
        o, S = _scan(leaves["q"], leaves["k"], leaves["v"], G, leaves["kappa"], scale, 32, S0_leaf)
    loss = (o * dO.to(dtype)).sum()
    if dS_T is not None:
        loss = loss + (S * dS_T.to(dtype)).sum()
    loss.backward()
    out = {"o": o.detach(), "S_T": S.detach(), "dg": G.grad.detach()}
    for name in ("q", "k", "v", "beta", "kappa"):
        if name in leaves:
            out["d" + name] = leaves[name].grad.detach()
    if S0_leaf is not None:
        out["dS0"] = S0_leaf.grad.detach()
    return out


def iso_gain_grads(a, omega, r, initial_precision, dgain, posterior_scale=1.0, dtype=torch.float64):
    """Autograd VJP of :func:`iso_gain`: ``(beta, da, domega, dr, d_initial_precision)``
    (the contract of ``_IsoKDNGainFunction.backward``, iso_kdn_chunk.py:1926-1963)."""
    la, lw, lr, lp = (t.detach().to(dtype).clone().requires_grad_(True) for t in (a, omega, r, initial_precision))
    beta, _, _ = iso_gain(la, lw, lr, lp, posterior_scale)
    (beta * dgain.to(dtype)).sum().backward()
    return beta.detach(), la.grad, lw.grad, lr.grad, lp.grad


def diag_gain_grads(k, alpha, omega, r, initial_precision, omega_raw, r_raw, dkappa, dtype=torch.float64):
    """VJP in the contract of ``_DiagKdnGainFunction.backward`` (diag_kdn_chunk.py:2700-2734):
    ``(kappa, dk, dalpha, domega_raw, dr_raw, d_initial_precision)``, where the
    omega and r cotangents leave through the softplus VJP ``* sigmoid(raw)``
    (diag_kdn_chunk.py:680-684)."""
    lk, la, lw, lr, lp = (
        t.detach().to(dtype).clone().requires_grad_(True) for t in (k, alpha, omega, r, initial_precision)
    )
    kappa, _ = diag_gain(lk, la, lw, lr, lp)
    (kappa * dkappa.to(dtype)).sum().backward()
    domega_raw = lw.grad * torch.sigmoid(omega_raw.to(dtype))
    dr_raw = lr.grad * torch.sigmoid(r_raw.to(dtype))
    return kappa.detach(), lk.grad, la.grad, domega_raw, dr_raw, lp.grad


# ----------------------------------------------------------------------------
# Seeded input generators (q, k ~ N(0,1) L2-normalised,
# v ~ N(0,1), ln(alpha) = -softplus(N(0,1)), beta = sigmoid(N(0,1)),
# omega = softplus(N(0,1)), r = 0.01 + softplus(N(0,1)), dO ~ N(0,1)).
# ----------------------------------------------------------------------------

def _softplus(x):
    return torch.nn.functional.softplus(x)


def make_iso_inputs(B, T, H, K=128, V=128, seed=0, dtype=torch.bfloat16, decay_scale=1.0):
    """Inputs of ``_chunk_kda_precumsum_paired`` and ``iso_kdn_gain`` on CPU.

    Draw order is fixed: q, k, v, x_alpha, x_beta, x_omega, x_r, dO.  q and k are
    drawn raw (the op normalises them); ``decay_scale`` multiplies ln(alpha)
    to exercise strong-decay chunks.
    """
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, K, generator=gen)
    k = torch.randn(B, T, H, K, generator=gen)
    v = torch.randn(B, T, H, V, generator=gen)
    log_alpha = -_softplus(torch.randn(B, T, H, K, generator=gen)) * decay_scale
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    omega = _softplus(torch.randn(B, T, H, generator=gen))
    r = 0.01 + _softplus(torch.randn(B, T, H, generator=gen))
    dO = torch.randn(B, T, H, V, generator=gen)
    g = g_cumsum_from_log_alpha(log_alpha, 64).float()
    a = torch.exp(2.0 * log_alpha).mean(-1)
    return {
        "q": q.to(dtype), "k": k.to(dtype), "v": v.to(dtype), "g_cumsum": g,
        "beta": beta, "a": a, "omega": omega, "r": r, "log_alpha": log_alpha,
        "dO": dO.to(dtype),
    }


def make_diag_inputs(B, T, H, K=128, V=128, seed=0, decay_scale=1.0):
    """Inputs of ``_diag_kdn_gain`` and ``chunk_kalman`` on CPU (config 2).

    Draw order: q, k, v, x_alpha, omega_raw, r_raw, dO.  q_memory and k_memory
    are the L2-normalised draws in bf16, k_gain the same keys in fp32;
    omega = softplus(omega_raw), r = 0.01 + softplus(r_raw) with the raw logits
    rounded to bf16 first (they are bf16 at the boundary); initial precision 1.
    """
    gen = torch.Generator().manual_seed(seed)
    q = l2norm(torch.randn(B, T, H, K, generator=gen))
    k = l2norm(torch.randn(B, T, H, K, generator=gen))
    v = torch.randn(B, T, H, V, generator=gen)
    log_alpha = -_softplus(torch.randn(B, T, H, K, generator=gen)) * decay_scale
    omega_raw = torch.randn(B, T, H, K, generator=gen).to(torch.bfloat16)
    r_raw = torch.randn(B, T, H, generator=gen).to(torch.bfloat16)
    dO = torch.randn(B, T, H, V, generator=gen)
    return {
        "q": q.to(torch.bfloat16), "k": k.to(torch.bfloat16), "v": v.to(torch.bfloat16),
        "k_gain": k.float(), "alpha": torch.exp(log_alpha), "log_alpha": log_alpha,
        "g_cumsum": g_cumsum_from_log_alpha(log_alpha, 32).float(),
        "omega_raw": omega_raw, "r_raw": r_raw,
        "omega": _softplus(omega_raw.float()), "r": 0.01 + _softplus(r_raw.float()),
        "initial_precision": torch.ones(H),
        "dO": dO,
    }


# ----------------------------------------------------------------------------
# Isotropic gate frontend (iso_kdn_chunk.py:740-953, the scalar preparation in
# front of the gain and the memory scan).  softplus is the definition the
# reference calls (flash-linear-attention 0.5.1, fla/ops/utils/softplus.py):
# x above 20, else ln(1 + e^x).
# ----------------------------------------------------------------------------

def _softplus_fla(x):
    return torch.where(x > 20.0, x, torch.log1p(torch.exp(torch.clamp(x, max=20.0))))


def iso_gate(g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, initial_precision_param, omega_min, r_min,
             chunk=64):
    """``(g_cumsum, a, omega, r, initial_precision)`` of the gate frontend
    (iso_kdn_chunk.py:786-814): g = -exp(A_log) softplus(g_raw + dt_bias), its
    chunk-local inclusive prefix times log2(e), a = mean_k exp(2 g), omega and r
    from the two halves of omega_r_raw, initial_precision = 0.1 + softplus."""
    B, T, H, K = g_raw.shape
    x = g_raw + dt_bias.view(1, 1, H, K)
    g = -torch.exp(A_log).view(1, 1, H, 1) * _softplus_fla(x)
    pad = (-T) % chunk
    gp = torch.nn.functional.pad(g, (0, 0, 0, 0, 0, pad))
    g_cumsum = gp.view(B, (T + pad) // chunk, chunk, H, K).cumsum(2).view(B, T + pad, H, K)[:, :T] / LN2
    a = torch.exp(2.0 * g).mean(-1)
    omega = omega_min + _softplus_fla(omega_r_raw[..., :H] + omega_bias)
    r = r_min + _softplus_fla(omega_r_raw[..., H:] + r_bias)
    initial_precision = 0.1 + _softplus_fla(initial_precision_param)
    return g_cumsum, a, omega, r, initial_precision


def iso_gate_grads(inputs, cotangents, omega_min, r_min, dtype=torch.float64):
    """Forward outputs and the seven parameter gradients of the gate frontend
    under the paired-cotangent contract (iso_kdn_chunk.py:817-953): the
    g_cumsum cotangent arrives as ``dg_pre_reverse`` in natural-log coordinates
    before the reverse chunk prefix, i.e. ``dL/dg_cumsum = ln(2) dg_pre``.
    ``inputs``: g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias,
    initial_precision_param; ``cotangents``: dg_pre_reverse, da, domega, dr,
    d_initial_precision (None = zero).  Returns (outputs, grads)."""
    leaves = [t.detach().to(dtype).clone().requires_grad_(True) for t in inputs]
    outs = iso_gate(*leaves, omega_min, r_min)
    loss = 0.0
    for i, (o, c) in enumerate(zip(outs, cotangents)):
        if c is None:
            continue
        c = c.to(dtype)
        if i == 0:
            c = c * LN2
        loss = loss + (o * c).sum()
    grads = torch.autograd.grad(loss, leaves, allow_unused=True)
    grads = [torch.zeros_like(l) if g is None else g for l, g in zip(leaves, grads)]
    return [o.detach() for o in outs], grads


DIAG_ALPHA_FLOOR = 1e-6


def diag_gate(retention_raw, omega_raw, r_raw, A_log, dt_bias, initial_precision_param, chunk=32):
    """``(g_cumsum, alpha, omega, r, initial_precision)`` of the diagonal
    frontend (diag_kdn_chunk.py:1867-1906 with OMEGA_COUPLING / EMIT_RAW_G off,
    omega_min 0, r_min 0.01, as launched at :2237): ell = -exp(A_log)
    softplus(retention_raw + dt_bias), alpha = exp(ell), g_cumsum = log2(e)
    times the 32-token-chunk inclusive prefix of ln max(alpha, 1e-6)."""
    B, T, H, K = retention_raw.shape
    x = retention_raw + dt_bias.view(1, 1, H, K)
    ell = -torch.exp(A_log).view(1, 1, H, 1) * _softplus_fla(x)
    alpha = torch.exp(ell)
    ell_mem = torch.log(torch.clamp(alpha, min=DIAG_ALPHA_FLOOR))
    pad = (-T) % chunk
    ep = torch.nn.functional.pad(ell_mem, (0, 0, 0, 0, 0, pad))
    g_cumsum = ep.view(B, (T + pad) // chunk, chunk, H, K).cumsum(2).view(B, T + pad, H, K)[:, :T] / LN2
    omega = _softplus_fla(omega_raw)
    r = 0.01 + _softplus_fla(r_raw)
    initial_precision = 0.1 + _softplus_fla(initial_precision_param)
    return g_cumsum, alpha, omega, r, initial_precision


def diag_gate_grads(inputs, cotangents, dtype=torch.float64):
    """Forward outputs and the six input gradients of the diagonal frontend
    under its paired-cotangent contract (diag_kdn_chunk.py:1969-2051,
    :2265-2443): the g_cumsum cotangent is reverse-prefixed without the log2(e)
    factor, i.e. ``dL/dg_cumsum = ln(2) d_g_cumsum``; the memory term is dropped
    where alpha is below the 1e-6 floor (the clamp's gradient).  ``inputs``:
    retention_raw, omega_raw, r_raw, A_log, dt_bias, initial_precision_param;
    ``cotangents``: d_g_cumsum, d_alpha, d_omega, d_r, d_initial_precision
    (None = zero).  Returns (outputs, grads)."""
    leaves = [t.detach().to(dtype).clone().requires_grad_(True) for t in inputs]
    outs = diag_gate(*leaves)
    loss = 0.0
    for i, (o, c) in enumerate(zip(outs, cotangents)):
        if c is None:
            continue
        c = c.to(dtype)
        if i == 0:
            c = c * LN2
        loss = loss + (o * c).sum()
    grads = torch.autograd.grad(loss, leaves, allow_unused=True)
    grads = [torch.zeros_like(l) if g is None else g for l, g in zip(leaves, grads)]
    return [o.detach() for o in outs], grads


def make_diag_gate_inputs(B, T, H, K=128, seed=0):
    """Seeded inputs (bf16 vectors, fp32 parameters, as the reference's
    validation requires) and fp32 cotangents of the diagonal frontend on CPU.
    A_log spans rates of about 1 to 20 and retention_raw has unit-2 spread, so
    some alphas fall below the 1e-6 floor."""
    gen = torch.Generator().manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=gen)  # noqa: E731
    dt = torch.exp(torch.rand(H, K, generator=gen) * (math.log(0.1) - math.log(0.001)) + math.log(0.001))
    inputs = (
        (n(B, T, H, K) * 2.0).to(torch.bfloat16),
        n(B, T, H, K).to(torch.bfloat16),
        n(B, T, H).to(torch.bfloat16),
        torch.log(torch.rand(H, generator=gen) * 19.0 + 1.0),
        dt + torch.log(-torch.expm1(-dt)),
        n(H),
    )
    cotangents = (n(B, T, H, K), n(B, T, H, K), n(B, T, H, K), n(B, T, H), n(H))
    return inputs, cotangents


def make_iso_gate_inputs(B, T, H, K=128, seed=0, g_dtype=torch.float32, wr_dtype=torch.float32):
    """Seeded inputs and cotangents of the gate frontend on CPU (fp32 unless
    the dtypes say otherwise; the parameters always fp32)."""
    gen = torch.Generator().manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=gen)  # noqa: E731
    inputs = (
        n(B, T, H, K).to(g_dtype),
        n(B, T, 2 * H).to(wr_dtype),
        n(H) * 0.5,
        n(H) * 0.5,
        n(H) * 0.5 - 1.0,
        n(H * K) * 0.5,
        n(H),
    )
    cotangents = (n(B, T, H, K), n(B, T, H), n(B, T, H), n(B, T, H), n(H))
    return inputs, cotangents


# ----------------------------------------------------------------------------
# Diagonal q / k normalisation (_diag_kdn_normalize, diag_kdn_chunk.py:2162;
# kernels :194 forward, :235 backward).  Unlike the recurrences above this is
# restated in float32 step by step, because the reference fixes every
# rounding: squares and sums in round-to-nearest fp32 in PyTorch's reduction
# order for a row held by one warp (lane l owns elements l, l+32, l+64, l+96:
# ((a0 + a1) + a2) + a3 for calls of >= 16 rows, (a0 + a2) + (a1 + a3) for
# fewer, :109-133; then a shuffle-down tree over the 32 lanes with offsets 1,
# 2, 4, 8, 16, :128-133), IEEE division and square root, round-to-nearest-even
# bf16 stores (:161-172).  Products and sums are single fp32 torch ops (one
# correctly rounded operation each); square roots and quotients are taken in
# float64 and rounded once to fp32, which gives the correctly rounded fp32
# result (53 >= 2 * 24 + 2 bits), whereas torch's vectorised fp32 sqrt on the
# CPU is not always correctly rounded.  The outputs are reproduced bit for bit.
# ----------------------------------------------------------------------------

def _sqrt_rn(x):
    return torch.sqrt(x.double()).float()


def _div_rn(a, b):
    return (a.double() / b.double()).float()

def _norm_lane_values(a, small_rows):
    """a [rows, 32, 4] per-lane terms -> [rows, 32] lane values."""
    f32 = torch.float32
    if small_rows:
        return (a[..., 0] + a[..., 2]).to(f32) + (a[..., 1] + a[..., 3]).to(f32)
    return ((a[..., 0] + a[..., 1]) + a[..., 2]) + a[..., 3]


def _norm_row_sum(a, small_rows):
    """The row total of per-lane terms a [rows, 32, 4] in the reference's order."""
    v = _norm_lane_values(a, small_rows)
    for off in (1, 2, 4, 8, 16):
        shifted = torch.cat((v[:, off:], v[:, 32 - off:]), 1)  # lanes past 31 keep their own value
        v = v + shifted
    return v[:, 0]


def _norm_lanes(x, K):
    """[rows, K] -> [rows, 32, 4] with lane l holding elements l + 32 j (zeros past K)."""
    rows = x.shape[0]
    out = torch.zeros(rows, 32, 4, dtype=torch.float32)
    out[..., :K // 32] = x.reshape(rows, K // 32, 32).transpose(1, 2)
    return out


def _norm_unlanes(y, K):
    return y[..., :K // 32].transpose(1, 2).reshape(y.shape[0], K)


def _norm_denominator(norm):
    return torch.where(torch.isnan(norm), norm, torch.clamp(norm, min=1e-12))


def diag_normalize(q_raw, k_raw):
    """``(q_memory bf16, k_gain fp32, k_memory bf16, q_norm, k_norm)`` of the
    diagonal boundary normalisation, bit-exact (float32 CPU restatement)."""
    shape = q_raw.shape
    K = shape[-1]
    rows = q_raw.numel() // K
    small = rows < 16
    outs = []
    for x in (q_raw, k_raw):
        xl = _norm_lanes(x.reshape(rows, K).float(), K)
        norm = _sqrt_rn(_norm_row_sum(xl * xl, small))
        d = _norm_denominator(norm)
        outs.append((_norm_unlanes(_div_rn(xl, d[:, None, None]), K).reshape(shape), norm.reshape(shape[:-1])))
    (qn, q_norm), (kn, k_norm) = outs
    return qn.to(torch.bfloat16), kn, kn.to(torch.bfloat16), q_norm, k_norm


def _norm_row_vjp(x, u, norm, small, K, out_dtype):
    rows = norm.shape[0]
    xl = _norm_lanes(x.reshape(rows, K).float(), K)
    ul = _norm_lanes(u.reshape(rows, K).float(), K)
    d = _norm_denominator(norm)[:, None, None]
    z = (-ul) * _div_rn(_div_rn(xl, d), d)
    g = _norm_row_sum(0.0 + z, small)[:, None, None]
    nrm = norm[:, None, None]
    unit = torch.where(nrm == 0, torch.zeros_like(xl), _div_rn(xl, torch.where(nrm == 0, torch.ones_like(nrm), nrm)))
    via = torch.where(nrm >= 1e-12, g * unit, torch.zeros_like(xl))
    total = _div_rn(ul, d) + via
    return _norm_unlanes(total, K).to(out_dtype)


def diag_normalize_backward(q_raw, k_raw, d_q_memory, d_k_gain, d_k_memory, q_norm, k_norm):
    """``(d_q_raw, d_k_raw)`` of :func:`diag_normalize` (None where no
    cotangent arrives), bit-exact: z = -u (x / d) / d, g = the ordered row sum
    of z, dx = u / d + g x / norm, rounded once to the input dtype
    (diag_kdn_chunk.py:174-191, :235-353)."""
    shape = q_raw.shape
    K = shape[-1]
    rows = q_raw.numel() // K
    small = rows < 16
    dq = dk = None
    if d_q_memory is not None:
        dq = _norm_row_vjp(q_raw, d_q_memory.float(), q_norm.reshape(rows).float(), small, K,
                           q_raw.dtype).reshape(shape)
    if d_k_gain is not None or d_k_memory is not None:
        if d_k_gain is not None and d_k_memory is not None:
            u = d_k_gain.float() + d_k_memory.float()
        else:
            u = (d_k_gain if d_k_gain is not None else d_k_memory).float()
        dk = _norm_row_vjp(k_raw, u, k_norm.reshape(rows).float(), small, K, k_raw.dtype).reshape(shape)
    return dq, dk


# ----------------------------------------------------------------------------
# Gated RMS normalisation of the scan output (the mixers' o_norm:
# flash-linear-attention's FusedRMSNormGated, lit_gpt/iso_kdn.py:192-197,
# 305-314; diag_kdn.py:216-221, 346-355): y = x rstd w act(g),
# rstd = 1 / sqrt(mean(x^2) + eps), act = sigmoid or g sigmoid(g).
# ----------------------------------------------------------------------------

def rms_norm_gated(x, g, weight, eps=1e-5, activation="sigmoid", dtype=torch.float64):
    """Forward in ``dtype`` (differentiable); weight may be None."""
    x, g = x.to(dtype), g.to(dtype)
    rstd = torch.rsqrt((x * x).mean(-1, keepdim=True) + eps)
    y = x * rstd
    if weight is not None:
        y = y * weight.to(dtype)
    s = torch.sigmoid(g)
    return y * (g * s if activation in ("swish", "silu") else s)


# ----------------------------------------------------------------------------
# Short causal depthwise convolution with SiLU (the mixers' q/k/v short
# convolution: qkv_causal_conv1d, iso_kdn_chunk.py:459; _fixed_short_conv,
# diag_kdn.py:75): y[t, c] = silu(sum_j w[c, j] x[t - W + 1 + j, c]).
# ----------------------------------------------------------------------------

def short_conv(x, weight, silu=True, dtype=torch.float64):
    """x [B, T, C], weight [C, W] -> [B, T, C] in ``dtype`` (differentiable)."""
    W = weight.shape[-1]
    xt = torch.nn.functional.pad(x.to(dtype).transpose(1, 2), (W - 1, 0))
    y = torch.nn.functional.conv1d(xt, weight.to(dtype).unsqueeze(1), groups=x.shape[-1]).transpose(1, 2)
    return torch.nn.functional.silu(y) if silu else y
