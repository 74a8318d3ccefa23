"""Collective microbenchmark: this package's peer-memory collectives against
NCCL on the same message, device-timed, max over ranks.

  reduce_scatter : every rank stores its W slices into the owners' receive
                   slots (push kernel), device barrier, owners sum their W slots
  all_gather     : every rank pushes its slice into every rank's output
  all_to_all     : every rank pushes slice j into rank j's receive slot

Only the data movement is timed here; in the optimizers the pushes are fused
into the producing GEMM's epilogue instead of a separate copy kernel.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m dion_b200.benchmarks.comm_bench [--mib 16,64,256]
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

from .. import ops
from ..parallel.symm import SymmetricHeap


def _time(fn, iters: int = 10, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--mib", default="16,64,256", help="per-rank input size (MiB of fp32)")
    a = p.parse_args(argv)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    rank, W = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    E = ops.ext()
    for mib in [int(x) for x in a.mib.split(",")]:
        n = (mib << 20) // 4 // W * W  # fp32 elements per rank, divisible by W
        x = torch.randn(n, device="cuda")
        chunk = n // W
        heap = SymmetricHeap(dist.group.WORLD, 2 * n * 4)
        recv = heap.view(0, (W, chunk), torch.float32)
        out_ag = heap.view(n * 4, (W, chunk), torch.float32)
        mine = torch.empty(chunk, device="cuda")
        # reduce-scatter: slice j -> rank j's slot [rank]
        rs_dst = [heap.ptr_tensor([heap.addr(j, rank * chunk * 4)]) for j in range(W)]
        # all-gather: my chunk -> every rank's out_ag[rank]
        order = [(rank + 1 + i) % W for i in range(W)]  # one source per destination at a time
        ag_dst = heap.ptr_tensor([heap.addr(j, n * 4 + rank * chunk * 4) for j in order])
        xs = x.view(W, chunk)

        def p2p_rs():
            for j in order:
                E.symm_push(xs[j], rs_dst[j])
            heap.barrier()
            E.symm_reduce_slots(recv, mine, W)

        def p2p_ag():
            E.symm_push(mine, ag_dst)
            heap.barrier()

        def p2p_a2a():
            for j in order:
                E.symm_push(xs[j], rs_dst[j])
            heap.barrier()

        nccl_out = torch.empty(chunk, device="cuda")
        full = torch.empty(n, device="cuda")
        a2a_out = torch.empty(n, device="cuda")
        res = {
            "rs_p2p_ms": _time(p2p_rs),
            "rs_nccl_ms": _time(lambda: dist.reduce_scatter_tensor(nccl_out, x)),
            "ag_p2p_ms": _time(p2p_ag),
            "ag_nccl_ms": _time(lambda: dist.all_gather_into_tensor(full, mine)),
            "a2a_p2p_ms": _time(p2p_a2a),
            "a2a_nccl_ms": _time(lambda: dist.all_to_all_single(a2a_out, x)),
        }
        # correctness of the P2P reduce-scatter against NCCL
        p2p_rs()
        dist.reduce_scatter_tensor(nccl_out, x)
        torch.cuda.synchronize()
        err = float((mine - nccl_out).abs().max())
        ops.check_status()
        if rank == 0:
            bytes_cross = n * 4 * (W - 1) / W  # per rank, each direction
            print(json.dumps({"world": W, "mib_per_rank": mib, **res, "rs_max_abs_err": err,
                              "rs_p2p_gbs_per_rank": bytes_cross / res["rs_p2p_ms"] / 1e6,
                              "rs_nccl_gbs_per_rank": bytes_cross / res["rs_nccl_ms"] / 1e6}), flush=True)
        heap.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
