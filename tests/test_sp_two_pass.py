"""Two-pass sequence parallelism (``kdn_b200.sequence_parallel``) on CPU ranks.

Each gloo rank runs ``diag_two_pass_forward`` / ``diag_two_pass_backward`` on
its contiguous segment with the float64 oracle standing in for the B200
passes (``tests/sp_oracle_segment.py``); the concatenated outputs and
gradients must equal one oracle graph over the whole sequence.  This checks
the segment summaries, the all-gathers, the prefix / suffix compositions of
the covariance maps, the state maps and their adjoints, and the prior's
gradient, all in exact (float64) arithmetic.  The composition helpers are
also checked against a direct sequential evaluation.  (The same driver on the
B200 kernels is checked by tests/test_gpu_sp_two_pass.py.)"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle

B, H, K, V, SEG = 1, 2, 16, 16, 64


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_inputs(T):
    gen = torch.Generator().manual_seed(11)
    sp = torch.nn.functional.softplus
    n = lambda *s: torch.randn(*s, generator=gen, dtype=torch.float64)  # noqa: E731
    la = -sp(n(B, T, H, K))
    return {
        "q": oracle.l2norm(n(B, T, H, K)), "k": oracle.l2norm(n(B, T, H, K)), "v": n(B, T, H, V),
        "g": oracle.g_cumsum_from_log_alpha(la, 32), "k_gain": oracle.l2norm(n(B, T, H, K)),
        "alpha": torch.exp(la - 0.05 * torch.rand(B, T, H, K, generator=gen, dtype=torch.float64)),
        "omega_raw": n(B, T, H, K), "r_raw": n(B, T, H), "prior": 0.5 + torch.rand(H, generator=gen,
                                                                                 dtype=torch.float64),
        "dO": n(B, T, H, V),
    }


NAMES = ("q", "k", "v", "g", "k_gain", "alpha", "omega_raw", "r_raw")


def _worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from kdn_b200.sequence_parallel import GroupComm, diag_two_pass_backward, diag_two_pass_forward
    from sp_oracle_segment import DiagSegmentOracle

    x = make_inputs(world * SEG)
    sl = slice(rank * SEG, (rank + 1) * SEG)
    s = {n: x[n][:, sl] for n in NAMES}
    seg = DiagSegmentOracle(s["q"], s["k"], s["v"], s["g"], s["k_gain"], s["alpha"], None, None, x["prior"],
                            s["omega_raw"], s["r_raw"], K ** -0.5)
    comm = GroupComm()
    o, phis = diag_two_pass_forward(seg, comm)
    grads = diag_two_pass_backward(seg, comm, phis, x["dO"][:, sl])
    torch.save({"o": o, **dict(zip(("dq", "dk", "dv", "dg", "dk_gain", "dalpha", "domega_raw", "dr_raw", "dprior"),
                                   grads))}, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def full_reference(x):
    L = {n: x[n].clone().requires_grad_(True) for n in NAMES + ("prior",)}
    omega = torch.nn.functional.softplus(L["omega_raw"])
    r = 0.01 + torch.nn.functional.softplus(L["r_raw"])
    kappa, _ = oracle.diag_gain(L["k_gain"], L["alpha"], omega, r, L["prior"])
    G = L["g"] * oracle.LN2
    G.retain_grad()
    am = oracle.alpha_from_g_cumsum(G, 32)
    S0 = torch.zeros(B, H, K, V, dtype=torch.float64)
    o, _ = oracle.memory_recurrence(L["q"], L["k"], L["v"], am, kappa, S0, K ** -0.5)
    (o * x["dO"]).sum().backward()
    ref = {"o": o.detach(), "dg": G.grad, "dprior": L["prior"].grad}
    ref.update({"d" + n: L[n].grad for n in NAMES if n != "g"})
    return ref


@pytest.mark.parametrize("world", [2, 3])
def test_two_pass_matches_full_sequence(world, tmp_path):
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    x = make_inputs(world * SEG)
    ref = full_reference(x)
    parts = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    errs = {}
    for key, full in ref.items():
        got = sum(p[key] for p in parts) if key == "dprior" else torch.cat([p[key] for p in parts], 1)
        errs[key] = ((got - full).abs().max() / full.abs().max()).item()
    # float64 throughout; the gate cotangent is a difference of neighbouring
    # tokens' retention terms and loses about eight digits to cancellation
    bad = {k: v for k, v in errs.items() if not v < (1e-7 if k == "dg" else 1e-9)}
    assert not bad, errs


ISO_NAMES = ("q", "k", "v", "g", "a", "omega", "r")


def make_iso_inputs(T):
    gen = torch.Generator().manual_seed(12)
    sp = torch.nn.functional.softplus
    n = lambda *s: torch.randn(*s, generator=gen, dtype=torch.float64)  # noqa: E731
    la = -sp(n(B, T, H, K))
    return {"q": n(B, T, H, K), "k": n(B, T, H, K), "v": n(B, T, H, V), "g": oracle.g_cumsum_from_log_alpha(la, 64),
            "a": torch.exp(2 * la).mean(-1), "omega": sp(n(B, T, H)), "r": 0.01 + sp(n(B, T, H)),
            "prior": 0.5 + torch.rand(H, generator=gen, dtype=torch.float64), "dO": n(B, T, H, V)}


def _iso_worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from kdn_b200.sequence_parallel import GroupComm, two_pass_backward, two_pass_forward
    from sp_oracle_segment import IsoSegmentOracle

    x = make_iso_inputs(world * SEG)
    sl = slice(rank * SEG, (rank + 1) * SEG)
    s = {n: x[n][:, sl] for n in ISO_NAMES}
    seg = IsoSegmentOracle(s["q"], s["k"], s["v"], s["g"], s["a"], s["omega"], s["r"], x["prior"], K ** -0.5, 0.5)
    comm = GroupComm()
    o, phis = two_pass_forward(seg, comm)
    grads = two_pass_backward(seg, comm, phis, x["dO"][:, sl])
    torch.save({"o": o, **dict(zip(("dq", "dk", "dv", "dg", "da", "domega", "dr", "dprior"), grads))},
               os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def iso_full_reference(x):
    L = {n: x[n].clone().requires_grad_(True) for n in ISO_NAMES + ("prior",)}
    beta, _, _ = oracle.iso_gain(L["a"], L["omega"], L["r"], L["prior"], 0.5)
    G = L["g"] * oracle.LN2
    G.retain_grad()
    qh, kh = oracle.l2norm(L["q"]), oracle.l2norm(L["k"])
    S0 = torch.zeros(B, H, K, V, dtype=torch.float64)
    o, _ = oracle.memory_recurrence(qh, kh, L["v"], oracle.alpha_from_g_cumsum(G, 64), beta[..., None] * kh, S0,
                                    K ** -0.5)
    (o * x["dO"]).sum().backward()
    ref = {"o": o.detach(), "dg": G.grad, "dprior": L["prior"].grad}
    ref.update({"d" + n: L[n].grad for n in ISO_NAMES if n != "g"})
    return ref


@pytest.mark.parametrize("world", [2, 3])
def test_iso_two_pass_matches_full_sequence(world, tmp_path):
    """The isotropic two-pass driver (scalar covariance maps, the same state
    maps) against one oracle graph over the whole sequence."""
    mp.spawn(_iso_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    x = make_iso_inputs(world * SEG)
    ref = iso_full_reference(x)
    parts = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    errs = {}
    for key, full in ref.items():
        got = sum(p[key] for p in parts) if key == "dprior" else torch.cat([p[key] for p in parts], 1)
        errs[key] = ((got - full).abs().max() / full.abs().max()).item()
    bad = {k: v for k, v in errs.items() if not v < (1e-7 if k == "dg" else 1e-9)}
    assert not bad, errs


def test_composition_helpers_match_sequential_evaluation():
    from kdn_b200.sequence_parallel import (carried_covariance, carried_covariance_adjoint, carried_state,
                                            carried_state_adjoint, mobius_apply)

    gen = torch.Generator().manual_seed(3)
    world = 4
    r = lambda *s: torch.rand(*s, generator=gen, dtype=torch.float64) + 0.5  # noqa: E731
    maps, p0 = r(world, 2, 3, 4), r(2, 3)
    phi, off, c = r(world, 2, 5, 5) / 5, r(world, 2, 5, 6), r(world, 2, 5, 6)
    adj = r(world, 2, 3, 2)
    p, S = p0, torch.zeros(2, 5, 6, dtype=torch.float64)
    for rank in range(world):
        assert torch.allclose(carried_covariance(maps, p0, rank), p)
        got = carried_state(phi, off, rank)
        assert (got is None and rank == 0) or torch.allclose(got, S)
        p, S = mobius_apply(maps[rank], p), phi[rank] @ S + off[rank]
    dS, lam = torch.zeros(2, 5, 6, dtype=torch.float64), torch.zeros(2, 3, dtype=torch.float64)
    for rank in range(world - 1, -1, -1):
        got = carried_state_adjoint(phi, c, rank)
        assert (got is None and rank == world - 1) or torch.allclose(got, dS)
        gl = carried_covariance_adjoint(adj, rank)
        assert (gl is None and rank == world - 1) or torch.allclose(gl, lam)
        dS, lam = phi[rank].transpose(-1, -2) @ dS + c[rank], adj[rank][..., 0] * lam + adj[rank][..., 1]
