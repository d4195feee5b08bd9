"""Worker for test_sp_nccl_two_gpus (run under torchrun): the isotropic KDN
scan of one sequence split over the ranks, state handed over with NCCL; rank 0
compares outputs and gradients with a single-GPU call on the whole sequence."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "kalman-delta-networks_b200")):
    sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import oracle  # noqa: E402
from kdn_b200.sequence_parallel import iso_segment, sp_iso_kdn  # noqa: E402


def main():
    out_dir = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", rank)
    T = 1024 * world
    d = oracle.make_iso_inputs(1, T, 4, seed=5)
    names = ("q", "k", "v", "g_cumsum", "a", "omega", "r")
    seg_len = T // world
    sl = slice(rank * seg_len, (rank + 1) * seg_len)
    L = {n: d[n][:, sl].contiguous().to(dev).requires_grad_(True) for n in names}
    P = torch.ones(4, device=dev, requires_grad=True)
    o = sp_iso_kdn(*(L[n] for n in names), P)
    o.backward(d["dO"][:, sl].to(dev))
    torch.cuda.synchronize()
    torch.save({"o": o.detach().cpu(), **{"d" + n: L[n].grad.cpu() for n in names}, "dprec": P.grad.cpu()},
               os.path.join(out_dir, f"sp{rank}.pt"))
    dist.barrier()
    if rank == 0:
        F = {n: d[n].to(dev).requires_grad_(True) for n in names}
        PF = torch.ones(4, device=dev, requires_grad=True)
        of, _, _ = iso_segment(*(F[n] for n in names), PF)
        of.backward(d["dO"].to(dev))
        parts = [torch.load(os.path.join(out_dir, f"sp{r}.pt")) for r in range(world)]

        def err(x, ref):
            x, ref = x.double(), ref.double().cpu()
            return ((x - ref).abs().max() / ref.abs().max()).item()

        errs = {"o": err(torch.cat([p["o"] for p in parts], 1), of.detach())}
        for n in names:
            errs["d" + n] = err(torch.cat([p["d" + n] for p in parts], 1), F[n].grad)
        errs["dprec"] = err(sum(p["dprec"] for p in parts), PF.grad)
        print("errors vs single GPU:", errs)
        assert all(v < 2e-2 for v in errs.values()), errs
        print("sp nccl ok")
    dist.barrier()
    diag_two_pass(rank, world, dev)
    dist.barrier()
    dist.destroy_process_group()


def diag_two_pass(rank, world, dev):
    """The diagonal KDN split over the ranks with the two-pass scheme (every
    rank at once, all-gathers over NCCL); every rank compares its slice with
    a single-GPU call on the whole sequence, which it evaluates itself."""
    from kdn_b200.diag_kdn_chunk import _diag_kdn_gain, chunk_kalman
    from kdn_b200.sequence_parallel import sp_diag_kdn_two_pass

    T, H, seg = 320 * world, 3, 320
    d = oracle.make_diag_inputs(1, T, H, seed=8)
    names = ("q", "k", "v", "g_cumsum", "k_gain", "alpha", "omega_raw", "r_raw", "initial_precision")
    F = {n: d[n].to(dev).requires_grad_(True) for n in names}
    kappa = _diag_kdn_gain(F["k_gain"], F["alpha"], d["omega"].to(dev), d["r"].to(dev), F["initial_precision"],
                           F["omega_raw"], F["r_raw"])
    of = chunk_kalman(F["q"], F["k"], kappa, F["v"], F["g_cumsum"], 128 ** -0.5)
    of.backward(d["dO"].to(dev))
    sl = slice(rank * seg, (rank + 1) * seg)
    S = {n: (d[n][:, sl] if d[n].dim() >= 3 else d[n]).contiguous().to(dev).requires_grad_(True) for n in names}
    o = sp_diag_kdn_two_pass(S["q"], S["k"], S["v"], S["g_cumsum"], S["k_gain"], S["alpha"],
                             d["omega"][:, sl].to(dev), d["r"][:, sl].to(dev), S["initial_precision"],
                             S["omega_raw"], S["r_raw"])
    o.backward(d["dO"][:, sl].to(dev))
    dprior = S["initial_precision"].grad.clone()
    dist.all_reduce(dprior)

    def err(x, ref):
        x, ref = x.double(), ref.double()
        return ((x - ref).abs().max() / ref.abs().max()).item()

    errs = {"o": err(o.detach(), of.detach()[:, sl]), "dprior": err(dprior, F["initial_precision"].grad)}
    for n in names[:-1]:
        errs["d" + n] = err(S[n].grad, F[n].grad[:, sl])
    worst = torch.tensor([max(errs.values())], device=dev)
    dist.all_reduce(worst, op=dist.ReduceOp.MAX)
    if rank == 0:
        print("two-pass diag errors vs single GPU (rank 0):", errs, "max over ranks:", worst.item())
    assert worst.item() < 2e-2, errs
    if rank == 0:
        print("sp two-pass nccl ok")


if __name__ == "__main__":
    main()
