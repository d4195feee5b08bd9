"""GPU parity at the benchmarked shapes (configs 1 and 2: B4 T4096 H18 d128).

The inputs come from ``bench.py``'s own generators, so the tiling checked
here (72 streams, 64 chunks per stream, H = 18 in the tensor maps' head
stride, thousands of CTAs per launch) is exactly the one the bench times.
The whole batch runs through the public operators, forward and backward;
the (b, h) streams are independent, so the float64 oracle is evaluated only
for a few sampled streams and compared with those slices of every output
and input gradient (and of the final state, from a continuation call).

Tolerances are the bf16 tensor-core path's (see ``test_gpu_parity.py``).
"""
import os

import pytest
import torch

import bench
import oracle
from kdn_b200 import _native as N
from kdn_b200 import _scan
from kdn_b200.diag_kdn_chunk import _diag_kdn_gain, chunk_kalman
from kdn_b200.iso_kdn_chunk import _chunk_kda_precumsum_paired, iso_kdn_gain

from test_gpu_parity import BF16_FTOL, BF16_TOL, check_errors

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
SAMPLES = ((0, 0), (1, 7), (3, 17))  # (b, h) streams compared with the oracle
D = 128


def streams(t):
    """[B, T, H, ...] -> [1, T, S, ...] for the sampled streams, float64 on the CPU."""
    return torch.stack([t[b, :, h] for b, h in SAMPLES], 1)[None].detach().double().cpu()


def test_iso_config1_sampled_streams():
    x = bench.make_iso(DEV, seed=1234)
    names = ("q", "k", "v", "g_cumsum", "a", "omega", "r", "prec")
    L = {n: x[n].detach().clone().requires_grad_(True) for n in names}
    beta = iso_kdn_gain(L["a"], L["omega"], L["r"], L["prec"], head_dim=D, out_dtype=torch.float32)
    o = _chunk_kda_precumsum_paired(q=L["q"], k=L["k"], v=L["v"], g_cumsum=L["g_cumsum"], beta=beta)
    o.backward(x["dO"])
    torch.cuda.synchronize()
    # the final state from the same kernels (continuation output of the forward)
    _, S_T, _ = _scan.scan_forward(N.KDN_ISO, x["q"], x["k"], x["v"], x["g_cumsum"], beta.detach(), D ** -0.5,
                                   want_final_state=True)

    # float64 oracle on the sampled streams: gain -> normalised keys -> memory recurrence
    R = {n: streams(x[n]).requires_grad_(True) for n in ("q", "k", "v", "a", "omega", "r")}
    G = (streams(x["g_cumsum"]) * oracle.LN2).requires_grad_(True)
    prec = torch.stack([x["prec"][h] for _, h in SAMPLES]).double().cpu()
    beta_r, _, _ = oracle.iso_gain(R["a"], R["omega"], R["r"], prec, 1.0)
    qh, kh = oracle.l2norm(R["q"]), oracle.l2norm(R["k"])
    alpha = oracle.alpha_from_g_cumsum(G, 64)
    S0 = torch.zeros(1, len(SAMPLES), D, D, dtype=torch.float64)
    o_r, S_r = oracle.memory_recurrence(qh, kh, R["v"], alpha, beta_r[..., None] * kh, S0, D ** -0.5)
    (o_r * streams(x["dO"])).sum().backward()

    got = {"o": streams(o), "S_T": torch.stack([S_T[b, h] for b, h in SAMPLES])[None].double().cpu(),
           "beta": streams(beta)}
    ref = {"o": o_r.detach(), "S_T": S_r.detach(), "beta": beta_r.detach()}
    for n in ("q", "k", "v", "a", "omega", "r"):
        got["d" + n], ref["d" + n] = streams(L[n].grad), R[n].grad
    got["dg"], ref["dg"] = streams(L["g_cumsum"].grad), G.grad
    bf16_typed = {"o", "dq", "dk", "dv"}
    check_errors("iso_config1", got, ref, bf16_typed, BF16_TOL, BF16_FTOL)


def test_diag_config2_sampled_streams():
    x = bench.make_diag(DEV, seed=1234)
    names = ("q", "k", "v", "g_cumsum", "k_gain", "alpha", "prec", "omega_raw", "r_raw")
    L = {n: x[n].detach().clone().requires_grad_(True) for n in names}
    kappa = _diag_kdn_gain(L["k_gain"], L["alpha"], x["omega"], x["r"], L["prec"], L["omega_raw"], L["r_raw"])
    o = chunk_kalman(L["q"], L["k"], kappa, L["v"], L["g_cumsum"], float(D ** -0.5))
    o.backward(x["dO"])
    torch.cuda.synchronize()
    _, S_T, _ = _scan.scan_forward(N.KDN_DIAG, x["q"], x["k"], x["v"], x["g_cumsum"], kappa.detach(), D ** -0.5,
                                   want_final_state=True)

    # the kernel rounds the fp32 cotangent to bf16 (diag_kdn_chunk.py:3277): the oracle gets the same one
    dO = streams(x["dO"].bfloat16())
    R = {n: streams(x[n]).requires_grad_(True) for n in ("q", "k", "v", "k_gain", "alpha", "omega_raw", "r_raw")}
    G = (streams(x["g_cumsum"]) * oracle.LN2).requires_grad_(True)
    prec = torch.stack([x["prec"][h] for _, h in SAMPLES]).double().cpu()
    omega = torch.nn.functional.softplus(R["omega_raw"])
    r = 0.01 + torch.nn.functional.softplus(R["r_raw"])
    kappa_r, _ = oracle.diag_gain(R["k_gain"], R["alpha"], omega, r, prec)
    alpha_mem = oracle.alpha_from_g_cumsum(G, 32)
    S0 = torch.zeros(1, len(SAMPLES), D, D, dtype=torch.float64)
    o_r, S_r = oracle.memory_recurrence(R["q"], R["k"], R["v"], alpha_mem, kappa_r, S0, D ** -0.5)
    (o_r * dO).sum().backward()

    got = {"o": streams(o), "S_T": torch.stack([S_T[b, h] for b, h in SAMPLES])[None].double().cpu(),
           "kappa": streams(kappa)}
    ref = {"o": o_r.detach(), "S_T": S_r.detach(), "kappa": kappa_r.detach()}
    for n in ("q", "k", "v", "k_gain", "alpha", "omega_raw", "r_raw"):
        got["d" + n], ref["d" + n] = streams(L[n].grad), R[n].grad
    got["dg"], ref["dg"] = streams(L["g_cumsum"].grad), G.grad
    bf16_typed = {"dq", "dk", "dv", "domega_raw", "dr_raw"}
    check_errors("diag_config2", got, ref, bf16_typed, BF16_TOL, BF16_FTOL)
