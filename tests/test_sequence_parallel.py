"""Sequence-parallel hand-off of the KDN state between ranks, on CPU (gloo).

Each rank runs its contiguous segment through ``kdn_b200.sequence_parallel.chain``
with the oracle as the segment compute; outputs and gradients of all ranks,
concatenated, must equal the oracle on the whole sequence.  This checks the
send/recv order, the carried states (memory S and covariance p) and their
cotangents in the backward.  (The B200 segment kernels are checked against
full-sequence calls in tests/test_gpu_parity.py.)"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle

B, T, H, K, V, SEG = 1, 192, 2, 16, 16, 64


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_inputs(variant):
    gen = torch.Generator().manual_seed(7)
    sp = torch.nn.functional.softplus
    x = {
        "q": torch.randn(B, T, H, K, generator=gen, dtype=torch.float64),
        "k": torch.randn(B, T, H, K, generator=gen, dtype=torch.float64),
        "v": torch.randn(B, T, H, V, generator=gen, dtype=torch.float64),
    }
    la = -sp(torch.randn(B, T, H, K, generator=gen, dtype=torch.float64))
    x["g"] = oracle.g_cumsum_from_log_alpha(la, 64 if variant == "iso" else 32)
    x["prec"] = 0.5 + torch.rand(H, generator=gen, dtype=torch.float64)
    x["r"] = 0.01 + sp(torch.randn(B, T, H, generator=gen, dtype=torch.float64))
    if variant == "iso":
        x["a"] = torch.exp(2 * la).mean(-1)
        x["omega"] = sp(torch.randn(B, T, H, generator=gen, dtype=torch.float64))
    else:
        x["kg"] = oracle.l2norm(x["k"])
        x["alpha"] = torch.exp(la)
        x["omega"] = sp(torch.randn(B, T, H, K, generator=gen, dtype=torch.float64))
    x["dO"] = torch.randn(B, T, H, V, generator=gen, dtype=torch.float64)
    return x


def iso_segment(q, k, v, g, a, omega, r, prec, S0, p0):
    beta, _, pT = oracle.iso_gain(a, omega, r, prec, 1.0, initial_covariance=p0)
    qh, kh = oracle.l2norm(q), oracle.l2norm(k)
    alpha = oracle.alpha_from_g_cumsum(g * oracle.LN2, 64)
    S0 = torch.zeros(q.shape[0], q.shape[2], K, V, dtype=q.dtype) if S0 is None else S0
    o, ST = oracle.memory_recurrence(qh, kh, v, alpha, beta[..., None] * kh, S0, K ** -0.5)
    return o, ST, pT


def diag_segment(q, k, v, g, kg, alpha_unused, omega, r, prec, S0, p0):
    alpha = oracle.alpha_from_g_cumsum(g * oracle.LN2, 32)
    kappa, pT = oracle.diag_gain(kg, alpha, omega, r, prec, initial_covariance=p0)
    S0 = torch.zeros(q.shape[0], q.shape[2], K, V, dtype=q.dtype) if S0 is None else S0
    o, ST = oracle.memory_recurrence(q, k, v, alpha, kappa, S0, K ** -0.5)
    return o, ST, pT


NAMES = {"iso": ("q", "k", "v", "g", "a", "omega", "r", "prec"),
         "diag": ("q", "k", "v", "g", "kg", "alpha", "omega", "r", "prec")}


def _worker(rank, world, port, variant, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from kdn_b200.sequence_parallel import Link, chain

    x = make_inputs(variant)
    sl = slice(rank * SEG, (rank + 1) * SEG)
    seg = {}
    for n in NAMES[variant]:
        t = x[n]
        t = t[:, sl] if t.dim() >= 3 else t
        seg[n] = t.clone().requires_grad_(True)
    cov_shape = (B, H) if variant == "iso" else (B, H, K)
    templates = [torch.empty(B, H, K, V, dtype=torch.float64), torch.empty(*cov_shape, dtype=torch.float64)]
    fn = iso_segment if variant == "iso" else diag_segment
    o = chain(fn, tuple(seg[n] for n in NAMES[variant]), templates, Link.from_group())
    (o * x["dO"][:, sl]).sum().backward()
    torch.save({"o": o.detach(), **{"d" + n: seg[n].grad for n in NAMES[variant]}},
               os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("variant", ["iso", "diag"])
def test_chain_matches_full_sequence(variant, tmp_path):
    world = T // SEG
    mp.spawn(_worker, args=(world, _free_port(), variant, str(tmp_path)), nprocs=world, join=True)
    x = make_inputs(variant)
    leaves = {n: x[n].clone().requires_grad_(True) for n in NAMES[variant]}
    fn = iso_segment if variant == "iso" else diag_segment
    o, _, _ = fn(*(leaves[n] for n in NAMES[variant]), None, None)
    (o * x["dO"]).sum().backward()
    parts = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    assert torch.allclose(torch.cat([p["o"] for p in parts], 1), o.detach(), rtol=1e-9, atol=1e-11)
    for n in NAMES[variant]:
        full = leaves[n].grad
        if full is None:
            continue
        if full.dim() >= 3:
            got = torch.cat([p["d" + n] for p in parts], 1)
        else:  # per-head prior: only rank 0's segment sees it
            got = sum(p["d" + n] for p in parts if p["d" + n] is not None)
        assert torch.allclose(got, full, rtol=1e-8, atol=1e-10), (n, (got - full).abs().max().item())
