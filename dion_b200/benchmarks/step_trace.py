"""Kernel timeline of one training step: torch.profiler trace plus a summary
of device time by owner (cuBLAS, cuDNN, this package's kernels, the rest)
and of the idle gaps between kernels.

    python -m dion_b200.benchmarks.step_trace --preset 1B --optimizer Muon \\
        --seq-len 4096 --local-batch 8 --out step_trace.json.gz

One process, one GPU; the trainer (FSDP2 over one rank, as in the 1B
benchmark) runs three warm-up steps, then one step under the profiler.
"""
from __future__ import annotations

import argparse
import collections
import gzip
import json
import os
import tempfile

import torch


def owner(name: str) -> str:
    n = name.lower()
    if name.startswith("nvjet") or "cublas" in n or "cutlass" in n:
        return "cuBLAS"
    if "cudnn" in n:
        return "cuDNN"
    if "bdion" in name:
        return "dion_b200"
    if "nccl" in n:
        return "NCCL"
    return "PyTorch"


def summarize(trace: dict, top: int = 25) -> dict:
    """Device time by owner and by kernel, span and idle time of a chrome trace."""
    k = sorted((e for e in trace["traceEvents"] if e.get("cat") == "kernel"), key=lambda e: e["ts"])
    if not k:
        return {"kernels": 0}
    by_owner, by_kernel = collections.Counter(), collections.Counter()
    end = k[0]["ts"]
    idle = 0.0
    for e in k:
        by_owner[owner(e["name"])] += e["dur"]
        by_kernel[(owner(e["name"]), e["name"][:100])] += e["dur"]
        if e["ts"] > end:
            idle += e["ts"] - end
        end = max(end, e["ts"] + e["dur"])
    span = end - k[0]["ts"]
    return {"kernels": len(k), "span_ms": span / 1e3, "busy_ms": sum(by_owner.values()) / 1e3, "idle_ms": idle / 1e3,
            "by_owner_ms": {o: v / 1e3 for o, v in by_owner.most_common()},
            "top_kernels_ms": [(o, n, v / 1e3) for (o, n), v in by_kernel.most_common(top)]}


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--preset", default="1B")
    p.add_argument("--optimizer", default="Muon")
    p.add_argument("--seq-len", type=int, default=4096)
    p.add_argument("--local-batch", type=int, default=8)
    p.add_argument("--out", default=None, help="write the chrome trace here (.json.gz)")
    a = p.parse_args(argv)
    from torch.profiler import ProfilerActivity, profile

    from ..integration.hybrid_optimizer import HybridOptimizersContainer
    from ..integration.trainer import Trainer, TrainerConfig

    oc = HybridOptimizersContainer.Config(name=a.optimizer, lr=0.02, weight_decay=0.01, scalar_lr=3e-4,
                                          scalar_beta1=0.9, scalar_beta2=0.95)
    tr = Trainer(TrainerConfig(model=a.preset, seq_len=a.seq_len, local_batch_size=a.local_batch, steps=10_000,
                               warmup_steps=200, seed=2, optimizer=oc))
    batches = [tr.data.next() for _ in range(4)]
    for t, l in batches[:3]:
        tr.train_step(t, l)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        tr.train_step(*batches[3])
        torch.cuda.synchronize()
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "trace.json")
        prof.export_chrome_trace(path)
        with open(path) as f:
            trace = json.load(f)
    if a.out:
        with gzip.open(a.out, "wt") as f:
            json.dump(trace, f)
    print(json.dumps(summarize(trace), indent=1))


if __name__ == "__main__":
    main()
