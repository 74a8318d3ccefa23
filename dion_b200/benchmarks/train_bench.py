"""Device-timed training-step benchmark for any model preset, optimizer and
(replicate x shard x TP) layout of the package's trainer.

The large-model runs (Llama-3 8B with Dion / AdaDionV2 adaptive rank under
FSDP, and Dion2 on an FSDP x TP mesh) go through this module; the 1B
headline stays in the repository's bench.py.

    python -m torch.distributed.run --nproc-per-node 4 -m dion_b200.benchmarks.train_bench \\
        --preset 8B --optimizer AdaDionV2 --dp-shard 4 --seq-len 8192 --local-batch 4 --steps 5 --warmup 3

Rank 0 prints one JSON line: whole-job tokens/s over the timed steps and the
mean optimizer-step time, both timed with CUDA events on the device and
taken as the max over ranks; synthetic uniform tokens from a fixed seed,
random init, bf16 compute with fp32 master weights (FSDP2 mixed precision).
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--preset", default="8B")
    p.add_argument("--optimizer", default="Dion", choices=["Muon", "Dion", "Dion2", "AdaDionV2", "AdamW"])
    p.add_argument("--dp-replicate", type=int, default=1)
    p.add_argument("--dp-shard", type=int, default=-1)
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--seq-len", type=int, default=8192)
    p.add_argument("--local-batch", type=int, default=4)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--ac", default="op", choices=["none", "op", "full"])
    p.add_argument("--rank-fraction", type=float, default=0.25, help="Dion rank; AdaDionV2 initial rank")
    p.add_argument("--rank-fraction-max", type=float, default=0.5, help="AdaDionV2 largest rank fraction")
    p.add_argument("--rank-min-fraction", type=float, default=1 / 16, help="AdaDionV2 smallest rank fraction")
    p.add_argument("--seed", type=int, default=3)
    p.add_argument("--lr", type=float, default=0.02)
    return p.parse_args(argv)


def _max_over_ranks(x: float) -> float:
    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def main(argv=None) -> None:
    a = parse(argv)
    from ..integration.hybrid_optimizer import HybridOptimizersContainer
    from ..integration.trainer import Trainer, TrainerConfig, clip_grad_norm_multi_mesh_

    from ..models.llama3 import llama3_config

    dim = llama3_config(a.preset).dim
    oc = HybridOptimizersContainer.Config(name=a.optimizer, lr=a.lr, weight_decay=0.01, scalar_lr=3e-4,
                                          rank_fraction=a.rank_fraction, rank_fraction_max=a.rank_fraction_max,
                                          init_rank_fraction=a.rank_fraction,
                                          rank_min=max(1, int(a.rank_min_fraction * dim)))
    cfg = TrainerConfig(model=a.preset, seq_len=a.seq_len, local_batch_size=a.local_batch, steps=10_000,
                        warmup_steps=100, seed=a.seed, dp_replicate=a.dp_replicate, dp_shard=a.dp_shard, tp=a.tp,
                        ac_mode="selective" if a.ac == "op" else a.ac, ac_option="op", optimizer=oc)
    tr = Trainer(cfg)
    world = dist.get_world_size() if dist.is_initialized() else 1
    dp = world // a.tp
    tokens_per_step = a.local_batch * a.seq_len * dp
    batches = [tr.data.next() for _ in range(a.warmup + a.steps)]
    dev = [(t.to(tr.device), l.to(tr.device)) for t, l in batches]
    params = list(tr.model.parameters())

    def step(tokens, labels, ev=None):
        tr._set_lr()
        loss = tr.forward_backward(tokens, labels)
        if tr.tp_mesh is not None:
            clip_grad_norm_multi_mesh_(params, 1.0, None)
        else:
            torch.nn.utils.clip_grad_norm_(params, 1.0, foreach=True)
        if ev is not None:
            ev[0].record()
        tr.optimizers.step()
        if ev is not None:
            ev[1].record()
        tr.optimizers.zero_grad(set_to_none=True)
        tr.step_idx += 1
        return loss

    for i in range(a.warmup):
        step(*dev[i])
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    opt_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    loss = None
    for i in range(a.steps):
        loss = step(*dev[a.warmup + i], ev=opt_ev[i])
    e.record()
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    ms = _max_over_ranks(s.elapsed_time(e))
    opt_ms = _max_over_ranks(sum(x.elapsed_time(y) for x, y in opt_ev) / a.steps)
    peak = _max_over_ranks(torch.cuda.max_memory_allocated() / 2**30)
    if not dist.is_initialized() or dist.get_rank() == 0:
        print(json.dumps({
            "metric": "training tokens/s + optimizer-step ms (device-timed, max over ranks)",
            "value": tokens_per_step * a.steps / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
            "ms_per_step": ms / a.steps, "optimizer_step_ms": opt_ms, "steps": a.steps, "warmup": a.warmup,
            "final_loss": float(loss.item()), "peak_mem_gib": peak,
            "config": {"model": f"llama3-{a.preset}", "optimizer": a.optimizer, "rank_fraction": a.rank_fraction,
                       "layout": {"dp_replicate": a.dp_replicate, "dp_shard": dp // a.dp_replicate, "tp": a.tp},
                       "seq_len": a.seq_len, "global_batch": a.local_batch * dp, "ac": a.ac,
                       "data": f"synthetic uniform tokens (seed {a.seed}), random init"},
        }), flush=True)
    from ..parallel.symm import release_all

    release_all()
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
