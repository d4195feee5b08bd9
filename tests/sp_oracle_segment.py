"""TEST INFRASTRUCTURE: the passes of ``kdn_b200.sequence_parallel.DiagSegmentB200``
evaluated by the float64 oracle, so the two-pass sequence-parallel driver
(``diag_two_pass_forward`` / ``diag_two_pass_backward``) can run on CPU ranks.

Every summary comes from the oracle's tokenwise recurrences
(``oracle.diag_gain``, ``oracle.memory_recurrence``; diag_kdn_naive.py:256-276,
479-500) and autograd: the composed covariance map from the per-token Moebius
maps p -> (a^2 p + omega) / (u a^2 p + 1 + u omega), u = K k^2 / r; the state
map as the state reached from the identity with zero values; the adjoint
summaries as gradients with a zero final cotangent.
"""
import torch

import oracle


class DiagSegmentOracle:
    def __init__(self, q, k, v, g_cumsum, k_gain, alpha, omega_unused, r_unused, prior, omega_raw, r_raw, scale):
        d = lambda t: t.detach().double().clone().requires_grad_(True)  # noqa: E731
        self.q, self.k, self.v, self.G = d(q), d(k), d(v), d(g_cumsum * oracle.LN2)
        self.k_gain, self.alpha, self.prior = d(k_gain), d(alpha), d(prior)
        self.omega_raw, self.r_raw = d(omega_raw), d(r_raw)
        self.B, self.T, self.H, self.K = q.shape
        self.V = v.shape[-1]
        self.scale = scale

    def _noise(self):
        return torch.nn.functional.softplus(self.omega_raw), 0.01 + torch.nn.functional.softplus(self.r_raw)

    def prior_covariance(self):
        return (1.0 / self.prior.detach()).view(1, self.H, 1).expand(self.B, self.H, self.K).contiguous()

    def cotangent(self, dO):
        return dO.double()

    def S_end_template(self):
        return self._f(self.B, self.H, self.K, self.V)

    def _f(self, *shape):
        return torch.zeros(*shape, dtype=torch.float64)

    def gain_maps(self):
        with torch.no_grad():
            omega, r = self._noise()
            M = torch.zeros(self.B, self.H, self.K, 2, 2, dtype=torch.float64)
            M[..., 0, 0] = M[..., 1, 1] = 1.0
            for t in range(self.T):
                a2 = self.alpha[:, t] ** 2
                w = omega[:, t]
                u = self.K * self.k_gain[:, t] ** 2 / r[:, t, :, None]
                Mt = torch.stack((torch.stack((a2, w), -1), torch.stack((u * a2, 1 + u * w), -1)), -2)
                M = Mt @ M
                M = M / M.abs().amax((-1, -2), keepdim=True)
            return M.reshape(self.B, self.H, self.K, 4)

    def gain_finish(self, p_in):
        self.p_in = (self.prior_covariance() if p_in is None else p_in.double()).clone().requires_grad_(True)
        self.first = p_in is None
        omega, r = self._noise()
        self.kappa, self.p_end = oracle.diag_gain(self.k_gain, self.alpha, omega, r, self.prior,
                                                  initial_covariance=self.p_in)
        self.kappa_leaf = self.kappa.detach().clone().requires_grad_(True)

    def scan_summary(self):
        with torch.no_grad():
            am = oracle.alpha_from_g_cumsum(self.G, 32)
            kap = self.kappa.detach()
            _, off = oracle.memory_recurrence(self.q, self.k, self.v, am, kap, self._f(self.B, self.H, self.K, self.V),
                                              self.scale)
            eye = torch.eye(self.K, dtype=torch.float64).expand(self.B, self.H, self.K, self.K)
            _, phi = oracle.memory_recurrence(self.q, self.k, torch.zeros(self.B, self.T, self.H, self.K,
                                                                          dtype=torch.float64),
                                              am, kap, eye.clone(), self.scale)
        return off, phi

    def scan_sequential(self, S_in):
        self.S_in = (self._f(self.B, self.H, self.K, self.V) if S_in is None else S_in.double()).clone()
        self.S_in.requires_grad_(True)
        am = oracle.alpha_from_g_cumsum(self.G, 32)
        self.o, self.S_end = oracle.memory_recurrence(self.q, self.k, self.v, am, self.kappa_leaf, self.S_in,
                                                      self.scale)
        return self.o.detach()

    def scan_adjoint_summary(self, dO):
        return torch.autograd.grad(self.o, self.S_in, dO.double(), retain_graph=True)[0]

    def scan_backward(self, dO, dS_end):
        outs, cots = [self.o], [dO.double()]
        if dS_end is not None:
            outs.append(self.S_end)
            cots.append(dS_end.double())
        dq, dk, dv, dG, self.dkappa = torch.autograd.grad(outs, [self.q, self.k, self.v, self.G, self.kappa_leaf],
                                                          cots, retain_graph=True)
        return dq, dk, dv, dG  # dG: the natural-log, pre-reverse gate cotangent, like the kernels' dg

    def gain_adjoint_summary(self):
        A = torch.autograd.grad(self.p_end, self.p_in, torch.ones_like(self.p_end), retain_graph=True)[0]
        Bc = torch.autograd.grad(self.kappa, self.p_in, self.dkappa, retain_graph=True)[0]
        return torch.stack((A, Bc), -1)

    def gain_backward(self, lam_end):
        outs, cots = [self.kappa], [self.dkappa]
        if lam_end is not None:
            outs.append(self.p_end)
            cots.append(lam_end.double())
        leaves = [self.k_gain, self.alpha, self.omega_raw, self.r_raw, self.prior, self.p_in]
        dk_gain, dalpha, domega_raw, dr_raw, dprior, dp_in = torch.autograd.grad(outs, leaves, cots,
                                                                                 allow_unused=True)
        dprior = torch.zeros_like(self.prior) if dprior is None else dprior
        if self.first:  # p_in = 1 / prior on the first segment
            dprior = dprior - (dp_in / self.prior.detach().view(1, self.H, 1) ** 2).sum((0, 2))
        return dk_gain, dalpha, domega_raw, dr_raw, dprior


class IsoSegmentOracle:
    """The passes of ``kdn_b200.sequence_parallel.IsoSegmentB200`` by the
    float64 oracle (``oracle.iso_gain``, ``oracle.memory_recurrence`` with
    L2-normalised q, k and kappa = beta k_hat; iso_kdn_naive.py:238-251,
    308-332): the per-token covariance map p -> r z / (r + s z), z = a p +
    omega, as the Moebius matrix [[r a, r omega], [s a, r + s omega]]."""

    def __init__(self, q, k, v, g_cumsum, a, omega, r, prior, scale, posterior_scale=1.0):
        d = lambda t: t.detach().double().clone().requires_grad_(True)  # noqa: E731
        self.q, self.k, self.v, self.G = d(q), d(k), d(v), d(g_cumsum * oracle.LN2)
        self.a, self.omega, self.r, self.prior = d(a), d(omega), d(r), d(prior)
        self.B, self.T, self.H, self.K = q.shape
        self.V = v.shape[-1]
        self.scale, self.s = scale, posterior_scale

    def _f(self, *shape):
        return torch.zeros(*shape, dtype=torch.float64)

    def prior_covariance(self):
        return (1.0 / self.prior.detach()).view(1, self.H).expand(self.B, self.H).contiguous()

    def cotangent(self, dO):
        return dO.double()

    def S_end_template(self):
        return self._f(self.B, self.H, self.K, self.V)

    def gain_maps(self):
        with torch.no_grad():
            M = torch.zeros(self.B, self.H, 2, 2, dtype=torch.float64)
            M[..., 0, 0] = M[..., 1, 1] = 1.0
            for t in range(self.T):
                a, w, r = self.a[:, t], self.omega[:, t], self.r[:, t]
                Mt = torch.stack((torch.stack((r * a, r * w), -1), torch.stack((self.s * a, r + self.s * w), -1)), -2)
                M = Mt @ M
                M = M / M.abs().amax((-1, -2), keepdim=True)
            return M.reshape(self.B, self.H, 4)

    def gain_finish(self, p_in):
        self.p_in = (self.prior_covariance() if p_in is None else p_in.double()).clone().requires_grad_(True)
        self.first = p_in is None
        self.beta, _, self.p_end = oracle.iso_gain(self.a, self.omega, self.r, self.prior, self.s,
                                                   initial_covariance=self.p_in)
        self.beta_leaf = self.beta.detach().clone().requires_grad_(True)

    def _scan(self, beta, v, S0):
        qh, kh = oracle.l2norm(self.q), oracle.l2norm(self.k)
        return oracle.memory_recurrence(qh, kh, v, oracle.alpha_from_g_cumsum(self.G, 64), beta[..., None] * kh, S0,
                                        self.scale)

    def scan_summary(self):
        with torch.no_grad():
            _, off = self._scan(self.beta.detach(), self.v, self._f(self.B, self.H, self.K, self.V))
            eye = torch.eye(self.K, dtype=torch.float64).expand(self.B, self.H, self.K, self.K).clone()
            _, phi = self._scan(self.beta.detach(), torch.zeros(self.B, self.T, self.H, self.K, dtype=torch.float64),
                                eye)
        return off, phi

    def scan_sequential(self, S_in):
        self.S_in = (self._f(self.B, self.H, self.K, self.V) if S_in is None else S_in.double()).clone()
        self.S_in.requires_grad_(True)
        self.o, self.S_end = self._scan(self.beta_leaf, self.v, self.S_in)
        return self.o.detach()

    def scan_adjoint_summary(self, dO):
        return torch.autograd.grad(self.o, self.S_in, dO.double(), retain_graph=True)[0]

    def scan_backward(self, dO, dS_end):
        outs, cots = [self.o], [dO.double()]
        if dS_end is not None:
            outs.append(self.S_end)
            cots.append(dS_end.double())
        dq, dk, dv, dG, self.dbeta = torch.autograd.grad(outs, [self.q, self.k, self.v, self.G, self.beta_leaf],
                                                         cots, retain_graph=True)
        return dq, dk, dv, dG

    def gain_adjoint_summary(self):
        A = torch.autograd.grad(self.p_end, self.p_in, torch.ones_like(self.p_end), retain_graph=True)[0]
        Bc = torch.autograd.grad(self.beta, self.p_in, self.dbeta, retain_graph=True)[0]
        return torch.stack((A, Bc), -1)

    def gain_backward(self, lam_end):
        outs, cots = [self.beta], [self.dbeta]
        if lam_end is not None:
            outs.append(self.p_end)
            cots.append(lam_end.double())
        leaves = [self.a, self.omega, self.r, self.prior, self.p_in]
        da, domega, dr, dprior, dp_in = torch.autograd.grad(outs, leaves, cots, allow_unused=True)
        dprior = torch.zeros_like(self.prior) if dprior is None else dprior
        if self.first:  # p_in = 1 / prior on the first segment
            dprior = dprior - (dp_in / self.prior.detach().view(1, self.H) ** 2).sum(0)
        return da, domega, dr, dprior
