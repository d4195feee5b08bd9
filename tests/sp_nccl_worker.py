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
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
