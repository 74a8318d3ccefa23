"""Distributed optimizer-step microbenchmark.

A stack of bf16 matrices (default: 48 of 4096x4096 and 48 of 4096x14336,
entries N(0, 1) from seed 1) sharded along dim 0 over the N ranks of a 1-D
mesh (FSDP2 layout). One step of
  * ``muon``: momentum, all-to-all to owners, 5 Newton-Schulz iterations with
    Keller Jordan's (3.4445, -4.7750, 2.0315), all-to-all back, update;
  * ``dion``: rank-1024 (fraction 1/4) power iteration, orthogonalisation,
    error feedback, update;
  * ``dion2``: top-L1 quarter of the rows of each momentum shard, rows sent
    to the matrix owner, Newton-Schulz, rows back, selective decay;
  * ``adadion_v2``: Dion with the adaptive rank schedule (effective rank of
    the column norms, one host read per shape group per step).
is timed on the device with CUDA events (max over ranks, mean over steps).

    python -m dion_b200.benchmarks.optimizer_bench --optimizer muon [--impl reference]
    torchrun --nproc-per-node 8 -m dion_b200.benchmarks.optimizer_bench ...

The reference arm runs the dion package's Muon (with its Keller-coefficient
Newton-Schulz from dion/muon_reference.py) or the reference's AdaDionV2
(non-adaptive = Dion) from baseline/_ref. Equivalent of the reference's
tier-B timer (ada_dion/benchmarks/tier_b_microbench.py:24-108), with device
timing instead of wall clock.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
import time

import torch
import torch.distributed as dist
from torch.distributed.device_mesh import init_device_mesh
from torch.distributed.tensor import Shard, distribute_tensor

HERE = os.path.dirname(os.path.abspath(__file__))
REF_PATH = os.path.join(os.path.dirname(os.path.dirname(HERE)), "baseline", "_ref")


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--optimizer", choices=["muon", "dion", "dion2", "adadion_v2"], default="muon")
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--n-square", type=int, default=48)
    p.add_argument("--n-wide", type=int, default=48)
    p.add_argument("--dim", type=int, default=4096)
    p.add_argument("--wide", type=int, default=14336)
    p.add_argument("--rank-fraction", type=float, default=0.25)
    p.add_argument("--replicated", action="store_true",
                   help="plain replicated tensors (DDP layout) instead of Shard(0) DTensors")
    p.add_argument("--trace", default=None,
                   help="after timing, profile one more step and write rank 0's kernel timeline (.json.gz)"
                        " plus a device-time summary line")
    return p.parse_args(argv)


def _init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if not dist.is_initialized():
        if world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1,
                                    device_id=torch.device("cuda", local))
    return dist.get_rank(), dist.get_world_size(), local


def build_params(args, mesh):
    shapes = [(args.dim, args.dim)] * args.n_square + [(args.dim, args.wide)] * args.n_wide
    gen = torch.Generator(device="cuda").manual_seed(1)
    params = []
    for shp in shapes:
        full = torch.randn(shp, device="cuda", generator=gen, dtype=torch.float32).to(torch.bfloat16)
        g = torch.randn(shp, device="cuda", generator=gen, dtype=torch.float32).to(torch.bfloat16)
        if args.replicated:
            p = torch.nn.Parameter(full.clone())
            p.grad = g.clone()
        else:
            p = torch.nn.Parameter(distribute_tensor(full, mesh, [Shard(0)]))
            p.grad = distribute_tensor(g, mesh, [Shard(0)])
        del full, g
        params.append(p)
    torch.cuda.empty_cache()
    return params


def build_optimizer(args, params, mesh, world):
    if args.impl == "ours":
        from dion_b200.optim import AdaDionV2, Dion, Dion2, Muon

        if args.optimizer == "muon":
            return Muon(params, distributed_mesh=mesh, lr=0.02, mu=0.95, weight_decay=0.01, ns_coeffs="keller")
        if args.optimizer == "dion2":
            return Dion2(params, distributed_mesh=mesh, lr=0.02, fraction=args.rank_fraction, weight_decay=0.01)
        if args.optimizer == "adadion_v2":
            return AdaDionV2(params, outer_shard_mesh=mesh, lr=0.02, mu=0.95, weight_decay=0.01,
                             adaptive_rank=True, rank_fraction_max=args.rank_fraction)
        return Dion(params, outer_shard_mesh=mesh, lr=0.02, mu=0.95, weight_decay=0.01,
                    rank_fraction=args.rank_fraction)
    sys.path.insert(0, REF_PATH)
    import torch._inductor.config as inductor_config

    if os.path.exists("/usr/bin/g++"):
        inductor_config.cpp.cxx = ("/usr/bin/g++",)
    if args.optimizer == "muon":
        from dion import Muon
        from dion.muon_reference import zeropower_via_newtonschulz5

        def keller(X, epsilon):
            return zeropower_via_newtonschulz5(X, eps=float(epsilon))

        return Muon(params, fsdp_mesh_dim=0, world_mesh=mesh, distributed_mesh=mesh, lr=0.02, mu=0.95,
                    weight_decay=0.01, newton_schulz_func=keller)
    from ada_dion.optim.adadion_v2 import AdaDionV2

    if args.optimizer == "adadion_v2":
        return AdaDionV2(params, outer_shard_mesh=mesh, lr=0.02, mu=0.95, weight_decay=0.01, adaptive_rank=True,
                         rank_fraction_max=args.rank_fraction)
    return AdaDionV2(params, outer_shard_mesh=mesh, lr=0.02, mu=0.95, weight_decay=0.01,
                     rank_fraction_max=args.rank_fraction)


def main(argv=None):
    args = parse(argv)
    if args.impl == "reference" and args.optimizer == "dion2":
        print(json.dumps({"metric": "optimizer_step_ms", "optimizer": "dion2", "impl": "reference",
                          "unavailable": "the reference environment has no Dion2 (dion.Dion2 is absent)"}))
        return
    rank, world, local = _init()
    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("dp_shard",))
    params = build_params(args, mesh)
    opt = build_optimizer(args, params, mesh, world)
    for _ in range(args.warmup):
        opt.step()
    torch.cuda.synchronize()
    dist.barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0 = time.perf_counter()
    for a, b in evs:
        a.record()
        opt.step()
        b.record()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1000 / args.steps
    ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    t = torch.tensor([ms, wall], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        print(json.dumps({
            "metric": "optimizer_step_ms", "optimizer": args.optimizer, "impl": args.impl, "n_gpus": world,
            "ms": float(t[0]), "wall_ms": float(t[1]), "steps": args.steps, "warmup": args.warmup,
            "matrices": f"{args.n_square}x{args.dim}^2 + {args.n_wide}x{args.dim}x{args.wide} bf16, "
                        + ("replicated" if args.replicated else "Shard(0)"),
            "p2p": os.environ.get("DION_B200_P2P", "1") != "0",
            "rank_fraction": args.rank_fraction if args.optimizer != "muon" else None,
        }))
    if args.trace:
        from torch.profiler import ProfilerActivity, profile

        from .step_trace import summarize

        dist.barrier()
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
            opt.step()
            torch.cuda.synchronize()
        if rank == 0:
            import gzip
            import tempfile

            with tempfile.TemporaryDirectory() as d:
                path = os.path.join(d, "t.json")
                prof.export_chrome_trace(path)
                with open(path) as f:
                    trace = json.load(f)
            with gzip.open(args.trace, "wt") as f:
                json.dump(trace, f)
            print(json.dumps({"trace_summary": summarize(trace, top=15)}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
