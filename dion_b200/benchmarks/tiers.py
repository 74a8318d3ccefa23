"""Benchmark tiers A (correctness), B (optimizer step timing: ``run_tier_b``
per matrix shape, and optimizer_bench.py for the distributed 96-matrix step)
and C (scale experiments), plus the profiler-trace parser.

Tier A: single-step invariants of every optimizer (finite, params move,
state keys), same-seed reproducibility and a distributed sanity run.
Tier C: torchrun command lines for FSDP at 8/16/32 GPUs, HSDP at 16/32 and a
performance-characterisation set (ada_dion/benchmarks/tier_c_scale.py:47-151).
``parse_profiler_trace`` sums collective time by kind from a Chrome trace,
like ada_dion/benchmarks/tier_b_microbench.py:157-217, and also reports this
package's kernels (``bdion::``) and the cuBLAS/cuDNN ones.

    python -m dion_b200.benchmarks.tiers a [--device cuda]
    python -m dion_b200.benchmarks.tiers b [--device cuda] [--warmup 10 --steps 100]
    python -m dion_b200.benchmarks.tiers c
    python -m dion_b200.benchmarks.tiers trace <trace.json>
"""
from __future__ import annotations

import argparse
import json
import math
from dataclasses import dataclass, field
from typing import Any, Dict, List

import torch

__all__ = ["run_tier_a", "run_tier_b", "TIER_B_SHAPES", "generate_c1_fsdp_experiments", "generate_c2_hsdp_experiments",
           "generate_performance_characterization", "experiment_to_cli", "parse_profiler_trace"]


def _optimizers():
    from ..optim import AGDion, AdaDion, AdaDionV2, Dion, Dion2, GSDion, Muon, QCDion, SDion

    small = dict(init_rank=8, rank_min=4, rank_max=32)
    return {
        "muon": lambda ps: Muon(ps, lr=0.02),
        "dion": lambda ps: Dion(ps, lr=0.02, rank_fraction=0.25),
        "dion2": lambda ps: Dion2(ps, lr=0.02, fraction=0.25),
        "adadion": lambda ps: AdaDion(ps, lr=0.02, **small),
        "adadion_v2": lambda ps: AdaDionV2(ps, lr=0.02, adaptive_rank=True, rank_min=4),
        "sdion": lambda ps: SDion(ps, lr=0.02, **small),
        "gsdion": lambda ps: GSDion(ps, lr=0.02, **small),
        "agdion": lambda ps: AGDion(ps, lr=0.02, **small),
        "qcdion": lambda ps: QCDion(ps, lr=0.02, **small),
    }


def _one_step(make, device, seed):
    torch.manual_seed(seed)
    ps = [torch.nn.Parameter(torch.randn(64, 32, device=device)), torch.nn.Parameter(torch.randn(32, 96, device=device))]
    before = [p.detach().clone() for p in ps]
    opt = make(ps)
    for p in ps:
        p.grad = torch.randn_like(p)
    opt.step()
    return ps, before, opt


def run_tier_a(device: str = "cpu") -> Dict[str, Dict[str, Any]]:
    """A1 invariants and A2 same-seed reproducibility for every optimizer."""
    out = {}
    for name, make in _optimizers().items():
        ps, before, opt = _one_step(make, device, 0)
        finite = all(bool(torch.isfinite(p).all()) for p in ps)
        moved = all(not torch.equal(p.detach(), b) for p, b in zip(ps, before))
        has_state = all(len(opt.state[p]) > 0 for p in ps)
        ps2, _, _ = _one_step(make, device, 0)
        repro = all(torch.equal(a.detach(), b.detach()) for a, b in zip(ps, ps2))
        out[name] = {"finite": finite, "params_changed": moved, "state_initialised": has_state,
                     "bit_exact_same_seed": repro, "pass": finite and moved and has_state and repro}
    return out


# ---------------------------------------------------------------- tier B
TIER_B_SHAPES = [(4096, 4096), (4096, 11008), (11008, 4096)]


def run_tier_b(device: str = "cuda", shapes=None, warmup: int = 10, steps: int = 100,
               dion_rank_fraction: float = 0.25, dion2_fraction: float = 0.25) -> Dict[str, Dict[str, Any]]:
    """``optimizer.step()`` alone on one bf16 matrix per shape, for AdamW,
    Muon, Dion and Dion2 (the reference's tier B, with its shapes, learning
    rates and step counts: ada_dion/benchmarks/tier_b_microbench.py:24-108).
    AdamW is this package's fused multi-tensor kernel (an ``algorithm:
    adamw`` group). On CUDA every step is timed with CUDA events; on CPU with
    the wall clock. Returns {"<m>x<n>": {optimizer: {mean_ms, std_ms, min_ms}}}."""
    from ..optim import Dion, Dion2, Muon

    configs = [
        ("AdamW", lambda ps: Muon([{"params": ps, "algorithm": "adamw"}], lr=3e-4, weight_decay=0.1)),
        ("Muon", lambda ps: Muon(ps, lr=0.02, mu=0.95)),
        ("Dion", lambda ps: Dion(ps, lr=0.02, rank_fraction=dion_rank_fraction)),
        ("Dion2", lambda ps: Dion2(ps, lr=0.02, fraction=dion2_fraction)),
    ]
    cuda = str(device).startswith("cuda")
    results: Dict[str, Dict[str, Any]] = {}
    for m, n in shapes or TIER_B_SHAPES:
        row = results.setdefault(f"{m}x{n}", {})
        for name, make in configs:
            torch.manual_seed(0)
            p = torch.nn.Parameter(torch.randn(m, n, device=device, dtype=torch.bfloat16))
            opt = make([p])
            times = []
            for i in range(warmup + steps):
                p.grad = torch.randn_like(p) * 0.01
                if cuda:
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    opt.step()
                    b.record()
                    b.synchronize()
                    t = a.elapsed_time(b)
                else:
                    import time

                    t0 = time.perf_counter()
                    opt.step()
                    t = (time.perf_counter() - t0) * 1e3
                opt.zero_grad(set_to_none=True)
                if i >= warmup:
                    times.append(t)
            mean = sum(times) / len(times)
            std = math.sqrt(sum((x - mean) ** 2 for x in times) / max(1, len(times) - 1))
            row[name] = {"mean_ms": mean, "std_ms": std, "min_ms": min(times)}
            del opt, p
    return results


# ---------------------------------------------------------------- tier C
@dataclass
class ExperimentConfig:
    name: str
    config_fn: str
    num_nodes: int = 1
    gpus_per_node: int = 8
    dp_shard: int = 8
    dp_replicate: int = 1
    tp_degree: int = 1
    steps: int = 1000
    extra: Dict[str, Any] = field(default_factory=dict)


OPTIMIZER_CONFIGS = {k: f"llama3_160m_{k}" for k in ("adamw", "muon", "dion", "dion2", "adadion")}


def generate_c1_fsdp_experiments(steps: int = 1000) -> List[ExperimentConfig]:
    out = []
    for gpus in (8, 16, 32):
        for opt, fn in OPTIMIZER_CONFIGS.items():
            out.append(ExperimentConfig(f"c1_fsdp{gpus}_{opt}", fn, num_nodes=max(1, gpus // 8),
                                        dp_shard=gpus, steps=steps))
    return out


def generate_c2_hsdp_experiments(steps: int = 1000) -> List[ExperimentConfig]:
    out = []
    for nodes in (2, 4):
        for opt, fn in OPTIMIZER_CONFIGS.items():
            out.append(ExperimentConfig(f"c2_hsdp{nodes}x8_{opt}", fn, num_nodes=nodes, dp_shard=8,
                                        dp_replicate=nodes, steps=steps))
    return out


def generate_performance_characterization(steps: int = 200) -> List[ExperimentConfig]:
    out = []
    for opt, fn in OPTIMIZER_CONFIGS.items():
        out.append(ExperimentConfig(f"perf_{opt}", fn, steps=steps,
                                    extra={"profiling.enable_profiling": "true",
                                           "profiling.save_traces_folder": f"traces/{opt}"}))
    return out


def experiment_to_cli(exp: ExperimentConfig) -> str:
    parts = ["torchrun", f"--nproc-per-node={exp.gpus_per_node}", f"--nnodes={exp.num_nodes}"]
    if exp.num_nodes > 1:
        parts += ["--node-rank=$NODE_RANK", "--rdzv-backend=c10d", '--rdzv-endpoint="$MASTER_ADDR:$MASTER_PORT"']
    else:
        parts += ["--master-addr 127.0.0.1", "--master-port ${PORT:-29500}"]
    parts += ["-m dion_b200.train", f"--config {exp.config_fn}", f"--training.steps {exp.steps}",
              f"--parallelism.data_parallel_shard_degree {exp.dp_shard}",
              f"--parallelism.data_parallel_replicate_degree {exp.dp_replicate}",
              f"--parallelism.tensor_parallel_degree {exp.tp_degree}"]
    parts += [f"--{k} {v}" for k, v in exp.extra.items()]
    return " \\\n    ".join(parts)


# ---------------------------------------------------------------- trace parser
def parse_profiler_trace(trace_path: str) -> Dict[str, Any]:
    """Aggregate device time from a PyTorch-profiler Chrome trace."""
    with open(trace_path) as f:
        trace = json.load(f)
    kinds = {"allreduce": ("allreduce", "all_reduce"), "allgather": ("allgather", "all_gather"),
             "reducescatter": ("reducescatter", "reduce_scatter"), "alltoall": ("alltoall", "all_to_all")}
    acc: Dict[str, List[float]] = {k: [0, 0.0] for k in list(kinds) + ["other"]}
    own = [0, 0.0]
    lib = [0, 0.0]
    for ev in trace.get("traceEvents", []):
        name = str(ev.get("name", "")).lower()
        dur = float(ev.get("dur", 0) or 0)
        if "nccl" in name:
            for k, keys in kinds.items():
                if any(s in name for s in keys):
                    acc[k][0] += 1
                    acc[k][1] += dur
                    break
            else:
                acc["other"][0] += 1
                acc["other"][1] += dur
        elif "bdion::" in name:
            own[0] += 1
            own[1] += dur
        elif "nvjet" in name or "cublas" in name or "cudnn" in name:
            lib[0] += 1
            lib[1] += dur
    res: Dict[str, Any] = {}
    total = 0.0
    for k, (c, us) in acc.items():
        res[f"nccl_{k}_count"] = int(c)
        res[f"nccl_{k}_ms"] = us / 1000
        total += us / 1000
    res["nccl_total_ms"] = total
    res["dion_b200_kernels_count"], res["dion_b200_kernels_ms"] = int(own[0]), own[1] / 1000
    res["library_kernels_count"], res["library_kernels_ms"] = int(lib[0]), lib[1] / 1000
    return res


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("tier", choices=["a", "b", "c", "trace"])
    p.add_argument("path", nargs="?")
    p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--steps", type=int, default=100)
    a = p.parse_args(argv)
    if a.tier == "a":
        res = run_tier_a(a.device)
        for k, v in res.items():
            print(f"{k:12s} {'PASS' if v['pass'] else 'FAIL'} {v}")
    elif a.tier == "b":
        print(json.dumps({"tier": "b", "device": a.device, "results": run_tier_b(a.device, warmup=a.warmup,
                                                                                steps=a.steps)}))
    elif a.tier == "c":
        for exp in generate_c1_fsdp_experiments() + generate_c2_hsdp_experiments() + \
                generate_performance_characterization():
            print(f"\n# {exp.name}\n{experiment_to_cli(exp)}")
    else:
        print(json.dumps(parse_profiler_trace(a.path), indent=1))


if __name__ == "__main__":
    main()
