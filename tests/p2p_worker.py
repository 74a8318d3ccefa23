"""Worker for tests/test_p2p_gpu.py: run under torchrun, one rank per GPU.

Runs Muon, Dion and Dion2 on Shard(0) DTensor parameters, and Muon on
replicated (DDP) parameters, twice: once with the in-kernel NVLink
collectives (symmetric peer memory) and once with NCCL collectives, from
identical seeds, and prints one JSON line per case with the largest
difference and the device time of a step on each path.
"""
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist
from torch.distributed.device_mesh import init_device_mesh
from torch.distributed.tensor import Shard, distribute_tensor

from dion_b200 import ops
from dion_b200.optim import Dion, Dion2, Muon

SHAPES = [(512, 256)] * 3 + [(256, 768)] * 2 + [(1024, 512)] * 4


def run(kind, mesh, p2p, steps, timed):
    os.environ["DION_B200_P2P"] = "1" if p2p else "0"
    torch.manual_seed(0)
    replicated = kind == "muon_ddp"

    def place(t):
        return t if replicated else distribute_tensor(t, mesh, [Shard(0)])

    params = [torch.nn.Parameter(place(torch.randn(s, device="cuda", dtype=torch.bfloat16) * 0.02))
              for s in SHAPES]
    if kind in ("muon", "muon_ddp"):
        opt = Muon(params, distributed_mesh=mesh, lr=0.02)
    elif kind == "dion2":
        opt = Dion2(params, distributed_mesh=mesh, lr=0.02, fraction=0.25)
    else:
        opt = Dion(params, outer_shard_mesh=mesh, lr=0.02, rank_fraction=0.25)
    ms = []
    for step in range(steps):
        torch.manual_seed(100 + step)
        for p in params:
            p.grad = place(torch.randn(p.shape, device="cuda", dtype=torch.bfloat16))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize()
        a.record()
        opt.step()
        b.record()
        torch.cuda.synchronize()
        ms.append(a.elapsed_time(b))
    t = torch.tensor([min(ms[-timed:])], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [(p.detach() if replicated else p.full_tensor()).float().cpu() for p in params], float(t)


def main():
    dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    rank = dist.get_rank()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    mesh = init_device_mesh("cuda", (dist.get_world_size(),))
    ok = True
    for kind in sys.argv[1:] or ["muon", "dion", "muon_ddp", "dion2"]:
        ref, t_nccl = run(kind, mesh, False, 4, 2)
        got, t_p2p = run(kind, mesh, True, 4, 2)
        diff = max(float((a - b).abs().max()) for a, b in zip(ref, got))
        scale = max(float(a.abs().max()) for a in ref)
        status = ops.ext().status_read()
        if rank == 0:
            print(json.dumps({"optimizer": kind, "world": dist.get_world_size(), "max_abs_diff": diff,
                              "max_abs": scale, "ms_nccl": t_nccl, "ms_p2p": t_p2p, "status": status}), flush=True)
        ok = ok and diff <= 1e-2 * max(scale, 1e-6) and status == 0
    from dion_b200.parallel.symm import _HEAPS, release_all

    canaries = all(h.check_canaries() for h in _HEAPS.values())  # all heaps of both paths
    if rank == 0:
        print(json.dumps({"canaries_intact": canaries, "heaps": len(_HEAPS)}), flush=True)
    ok = ok and canaries
    release_all()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
