"""Two-pass sequence parallelism on the B200 kernels, ranks emulated on one GPU.

Each emulated rank is a host thread that runs ``diag_two_pass_forward`` /
``diag_two_pass_backward`` (kdn_b200.sequence_parallel) on its contiguous
segment through the C ABI's split gain phases and partial scan modes; the
all-gather is a host barrier (every thread synchronises the device first), so
no kernel ever waits for another.  The concatenated outputs and gradients
must match the float64 oracle over the whole sequence within the bf16
tensor-core tolerance.  The same driver over NCCL between GPUs runs in
tests/sp_nccl_worker.py (two GPUs) and in bench.py's ``sp`` record.
"""
import threading

import pytest
import torch

import oracle
from kdn_b200.sequence_parallel import DiagSegmentB200, IsoSegmentB200, diag_two_pass_backward, diag_two_pass_forward

from test_gpu_parity import BF16_FTOL, BF16_TOL, check_errors

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
K = 128


class ThreadComm:
    """All-gather among host threads of one process (one emulated rank each)."""

    def __init__(self, rank, world, shared):
        self.rank, self.world, self.shared = rank, world, shared

    def all_gather(self, t):
        torch.cuda.synchronize()
        self.shared["slots"][self.rank] = t
        self.shared["barrier"].wait()
        out = torch.stack(self.shared["slots"])
        self.shared["barrier"].wait()  # every rank has read the slots before they are reused
        return out


def diag_segment(d, sl):
    t = {n: d[n][:, sl].contiguous().to(DEV) for n in
         ("q", "k", "v", "g_cumsum", "k_gain", "alpha", "omega", "r", "omega_raw", "r_raw")}
    return DiagSegmentB200(t["q"], t["k"], t["v"], t["g_cumsum"], t["k_gain"], t["alpha"], t["omega"], t["r"],
                           d["initial_precision"].to(DEV), t["omega_raw"], t["r_raw"], K ** -0.5)


def iso_segment(d, sl):
    t = {n: d[n][:, sl].contiguous().to(DEV) for n in ("q", "k", "v", "g_cumsum", "a", "omega", "r")}
    return IsoSegmentB200(t["q"], t["k"], t["v"], t["g_cumsum"], t["a"], t["omega"], t["r"],
                          d["initial_precision"].to(DEV), K ** -0.5, 1.0)


def run_ranks(world, d, seg_len, make_segment=diag_segment):
    shared = {"slots": [None] * world, "barrier": threading.Barrier(world, timeout=120)}
    results, errors = [None] * world, []

    def rank_main(rank):
        try:
            sl = slice(rank * seg_len, (rank + 1) * seg_len)
            seg = make_segment(d, sl)
            comm = ThreadComm(rank, world, shared)
            o, phis = diag_two_pass_forward(seg, comm)
            grads = diag_two_pass_backward(seg, comm, phis, d["dO"][:, sl].to(DEV))
            torch.cuda.synchronize()
            results[rank] = (o, grads)
        except BaseException as e:  # noqa: BLE001 - reported below; the barrier breaks the other ranks
            errors.append(e)
            shared["barrier"].abort()

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(world)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    if errors:
        raise errors[0]
    return results


@pytest.mark.parametrize("world,seg_len", [(2, 288), (4, 256)])
def test_two_pass_on_b200_matches_oracle(world, seg_len):
    T, H = world * seg_len, 2
    d = oracle.make_diag_inputs(1, T, H, seed=world + 40)
    d["dO"] = d["dO"].bfloat16().float()  # chunk_kalman rounds its cotangent to bf16
    parts = run_ranks(world, d, seg_len)
    names = ("dq", "dk", "dv", "dg", "dk_gain", "dalpha", "domega_raw", "dr_raw")
    got = {"o": torch.cat([p[0] for p in parts], 1)}
    for i, n in enumerate(names):
        got[n] = torch.cat([p[1][i] for p in parts], 1)
    got["dprior"] = sum(p[1][8] for p in parts)

    L = {n: d[n].double().clone().requires_grad_(True)
         for n in ("q", "k", "v", "k_gain", "alpha", "omega_raw", "r_raw", "initial_precision")}
    G = (d["g_cumsum"].double() * oracle.LN2).requires_grad_(True)
    omega = torch.nn.functional.softplus(L["omega_raw"])
    r = 0.01 + torch.nn.functional.softplus(L["r_raw"])
    kappa, _ = oracle.diag_gain(L["k_gain"], L["alpha"], omega, r, L["initial_precision"])
    S0 = torch.zeros(1, H, K, K, dtype=torch.float64)
    o, _ = oracle.memory_recurrence(L["q"], L["k"], L["v"], oracle.alpha_from_g_cumsum(G, 32), kappa, S0, K ** -0.5)
    (o * d["dO"].double()).sum().backward()
    ref = {"o": o.detach(), "dg": G.grad, "dprior": L["initial_precision"].grad}
    for n in ("q", "k", "v", "k_gain", "alpha", "omega_raw", "r_raw"):
        ref["d" + n] = L[n].grad
    check_errors(f"sp_two_pass_world{world}", got, ref, {"dq", "dk", "dv", "domega_raw", "dr_raw"}, BF16_TOL,
                 BF16_FTOL)


@pytest.mark.parametrize("world,seg_len", [(2, 320), (3, 192)])
def test_iso_two_pass_on_b200_matches_oracle(world, seg_len):
    """The isotropic segments (split scalar gain phases, the same scan modes)."""
    T, H = world * seg_len, 2
    d = oracle.make_iso_inputs(1, T, H, seed=world + 50, dtype=torch.bfloat16)
    d["initial_precision"] = torch.tensor([1.0, 0.7])
    parts = run_ranks(world, d, seg_len, iso_segment)
    names = ("dq", "dk", "dv", "dg", "da", "domega", "dr")
    got = {"o": torch.cat([p[0] for p in parts], 1)}
    for i, n in enumerate(names):
        got[n] = torch.cat([p[1][i] for p in parts], 1)
    got["dprior"] = sum(p[1][7] for p in parts)

    L = {n: d[n].double().clone().requires_grad_(True) for n in ("q", "k", "v", "a", "omega", "r")}
    P = d["initial_precision"].double().clone().requires_grad_(True)
    G = (d["g_cumsum"].double() * oracle.LN2).requires_grad_(True)
    beta, _, _ = oracle.iso_gain(L["a"], L["omega"], L["r"], P, 1.0)
    qh, kh = oracle.l2norm(L["q"]), oracle.l2norm(L["k"])
    S0 = torch.zeros(1, H, K, K, dtype=torch.float64)
    o, _ = oracle.memory_recurrence(qh, kh, L["v"], oracle.alpha_from_g_cumsum(G, 64), beta[..., None] * kh, S0,
                                    K ** -0.5)
    (o * d["dO"].double()).sum().backward()
    ref = {"o": o.detach(), "dg": G.grad, "dprior": P.grad}
    for n in ("q", "k", "v", "a", "omega", "r"):
        ref["d" + n] = L[n].grad
    check_errors(f"sp_iso_two_pass_world{world}", got, ref, {"o", "dq", "dk", "dv"}, BF16_TOL, BF16_FTOL)
