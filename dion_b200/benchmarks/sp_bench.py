"""Sequence-parallel TP collectives fused into the GEMMs vs the same GEMMs
around NCCL collectives, with the roofline of each.

    python -m torch.distributed.run --nproc-per-node 2 -m dion_b200.benchmarks.sp_bench \\
        --tokens 32768 --dim 4096 --hidden 14336

Times (CUDA events, max over ranks) one forward + backward of the MLP
sublayer's TP linears on a [tokens / T, dim] shard: all-gather -> w1, w3
(column-parallel) -> w2 (row-parallel) -> reduce-scatter, first on the
peer-memory path (parallel/sp.py), then with ``DION_B200_P2P=0``-style NCCL
collectives. Roofline = the slower of (GEMM FLOPs / measured bf16 peak) and
(bytes each GPU must send over NVLink / 770 GB/s per direction).
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from ..parallel.sp import SPGroup, sp_column_linears, sp_row_linear

NVLINK_GBS = 770.0  # measured peer copy per direction on B200 (NVLink 5)


def _peak_tflops() -> float:
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


def run(sp: SPGroup, x, w1, w3, w2, steps: int, warmup: int) -> float:
    def once():
        xs = x.detach().requires_grad_()
        a, b = sp_column_linears(sp, xs, [w1, w3])
        y = sp_row_linear(sp, torch.nn.functional.silu(a) * b, w2)
        y.backward(torch.ones_like(y))

    for _ in range(warmup):
        once()
    dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        once()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / steps], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", type=int, default=32768)
    p.add_argument("--dim", type=int, default=4096)
    p.add_argument("--hidden", type=int, default=14336)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    a = p.parse_args(argv)
    dist.init_process_group("nccl")
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    T, me = dist.get_world_size(), dist.get_rank()
    g = torch.Generator(device="cuda").manual_seed(0)
    n, D, H = a.tokens // T, a.dim, a.hidden // T
    x = torch.randn(n, D, device="cuda", dtype=torch.bfloat16, generator=g)
    w1 = (torch.randn(H, D, device="cuda", generator=g) * D ** -0.5).bfloat16().requires_grad_()
    w3 = (torch.randn(H, D, device="cuda", generator=g) * D ** -0.5).bfloat16().requires_grad_()
    w2 = (torch.randn(D, H, device="cuda", generator=g) * H ** -0.5).bfloat16().requires_grad_()
    res = {}
    for name, p2p in (("peer_memory", True), ("nccl", False)):
        sp = SPGroup(dist.group.WORLD, torch.device("cuda"))
        sp.p2p = sp.p2p and p2p
        res[name] = run(sp, x, w1, w3, w2, a.steps, a.warmup)
        res[name + "_path_active"] = sp.p2p
    N = a.tokens
    # forward 3 GEMMs + backward 6 GEMMs, each 2 * N * D * H flops on this rank
    flops = 9 * 2 * N * D * H
    # NVLink bytes sent per GPU: forward AG (bf16) + RS (fp32 partials), backward AG of x and dy
    # (bf16) + RS (fp32): every collective moves (T-1)/T of an [N, D] tensor
    frac = (T - 1) / T
    nv_bytes = frac * N * D * (2 + 4 + 2 + 2 + 4)
    roof_ms = max(flops / (_peak_tflops() * 1e12), nv_bytes / (NVLINK_GBS * 1e9)) * 1e3
    if me == 0:
        print(json.dumps({"metric": "sp_mlp_fwd_bwd_ms", "n_gpus": T, "tokens": N, "dim": D, "hidden": a.hidden,
                          "ms": res, "roofline_ms": roof_ms,
                          "fraction_of_roofline": {k: roof_ms / v for k, v in res.items()
                                                   if isinstance(v, float)}}), flush=True)
    from ..parallel.symm import release_all

    release_all()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
