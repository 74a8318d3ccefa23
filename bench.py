"""Headline benchmark: Llama-3 1B training step, Muon on the matrices + AdamW
on embeddings / norms / LM head, FSDP2 over N GPUs (one process per GPU),
synthetic uniform tokens (seed 2), random init, bf16 compute with fp32
master weights and optimizer state.

  python bench.py --gpus N --steps K --warmup W [--impl ours|reference]
                  [--optimizer muon|dion]

Rank 0 prints one JSON line. ``value`` is whole-job tokens/s over the K
timed steps (device-timed with CUDA events, max over ranks, inputs already
on the device); ``e2e`` is the same steps driven through the public
``Trainer.train_step`` API with the host->device copy of every step's
tokens from pinned memory and a device->host read of every step's loss.
``optimizer_step_ms`` is the device time of ``optimizer.step()`` (max over
ranks, mean over the timed steps).

``--impl reference`` runs the unmodified reference package installed in
baseline/_ref (its param grouping and the dion Muon / AdaDionV2 optimizer it
depends on) on torchtitan's own Llama-3 model, with the same FSDP2 plumbing,
data and timing.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
REF_PATH = os.path.join(HERE, "baseline", "_ref")

MODEL = dict(name="llama3-1B", dim=2048, n_layers=16, n_heads=32, n_kv_heads=8, ffn_dim=8192, vocab=128256)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--optimizer", choices=["muon", "dion"], default="muon")
    p.add_argument("--seq-len", type=int, default=4096)
    p.add_argument("--local-batch", type=int, default=8)
    p.add_argument("--no-e2e", action="store_true")
    return p.parse_args()


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons every 200 ms (rank 0)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", ",".join(str(g) for g in self.gpus)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- helpers
def max_over_ranks(x: float) -> float:
    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def barrier_sync():
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()


def make_batches(n, vocab, seq, lb, rank, world, seed):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        full = torch.randint(0, vocab, (lb * world, seq + 1), generator=g)
        mine = full[rank * lb:(rank + 1) * lb]
        out.append((mine[:, :-1].contiguous().pin_memory(), mine[:, 1:].contiguous().pin_memory()))
    return out


# ---------------------------------------------------------------- arms
def build_ours(args, world):
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    oc = HybridOptimizersContainer.Config(name="Muon" if args.optimizer == "muon" else "Dion", lr=0.02,
                                          weight_decay=0.01, scalar_lr=3e-4, scalar_beta1=0.9, scalar_beta2=0.95)
    cfg = TrainerConfig(model="1B", seq_len=args.seq_len, local_batch_size=args.local_batch, steps=10_000,
                        warmup_steps=200, seed=2, optimizer=oc)
    tr = Trainer(cfg)

    def step_device(tokens, labels, timers=None):
        tr._set_lr()
        loss = tr.forward_backward(tokens, labels)
        torch.nn.utils.clip_grad_norm_(tr.model.parameters(), 1.0, foreach=True)
        if timers is not None:
            timers[0].record()
        tr.optimizers.step()
        if timers is not None:
            timers[1].record()
        tr.optimizers.zero_grad(set_to_none=True)
        tr.step_idx += 1
        return loss

    def step_e2e(tokens_host, labels_host):
        return tr.train_step(tokens_host, labels_host).item()

    return step_device, step_e2e


def build_reference(args, world, mesh):
    """The reference's stock pieces: torchtitan Llama-3, FSDP2, ada_dion's
    param grouping and the optimizer it routes to (dion.Muon / AdaDionV2)."""
    sys.path.insert(0, REF_PATH)
    import torch._inductor.config as inductor_config
    import torch.nn.functional as F

    # the reference's torch.compile'd optimizer code also compiles small CPU
    # graphs; point Inductor at the system C++ compiler, whose OpenMP runtime
    # is installed on this image (the default one on PATH lacks libgomp.spec)
    if os.path.exists("/usr/bin/g++"):
        inductor_config.cpp.cxx = ("/usr/bin/g++",)
    from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard
    from torchtitan.models.llama3.model.args import TransformerModelArgs
    from torchtitan.models.llama3.model.model import Transformer
    from ada_dion.integration.param_grouper import group_params_for_hybrid

    margs = TransformerModelArgs(dim=MODEL["dim"], n_layers=MODEL["n_layers"], n_heads=MODEL["n_heads"],
                                 n_kv_heads=MODEL["n_kv_heads"], vocab_size=MODEL["vocab"], multiple_of=256,
                                 ffn_dim_multiplier=1.5, rope_theta=500000, max_seq_len=args.seq_len)
    torch.manual_seed(2)
    with torch.device("cuda"):
        model = Transformer(margs)
        model.init_weights()
    mp = MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32)
    blocks = list(model.layers.values())
    for i, b in enumerate(blocks):
        fully_shard(b, mesh=mesh, mp_policy=mp, reshard_after_forward=i < len(blocks) - 1)
    fully_shard(model, mesh=mesh, mp_policy=mp)

    g = group_params_for_hybrid(model)
    scalar = dict(algorithm="adamw", beta1=0.9, beta2=0.95, epsilon=1e-8)
    groups = [{"params": g.matrix_params}]
    groups.append({"params": g.embed_params, "lr": 3e-4, "weight_decay": 0.01, **scalar})
    groups.append({"params": g.output_params, "lr": 3e-4 / math.sqrt(MODEL["dim"]), "weight_decay": 0.01, **scalar})
    groups.append({"params": g.norm_params, "lr": 3e-4, "weight_decay": 0.0, **scalar})
    if args.optimizer == "muon":
        from dion import Muon

        opt = Muon(groups, fsdp_mesh_dim=0, world_mesh=mesh, distributed_mesh=mesh, lr=0.02, mu=0.95,
                   weight_decay=0.01, nesterov=False, adjust_lr="spectral_norm")
    else:
        from ada_dion.optim.adadion_v2 import AdaDionV2

        for gr in groups[1:]:
            gr["epsilon"] = 1e-8
        opt = AdaDionV2(groups, outer_shard_mesh=mesh if world > 1 else None, lr=0.02, rank_fraction_max=0.25,
                        weight_decay=0.01)
    base = [gr["lr"] for gr in opt.param_groups]
    state = {"step": 0}

    def set_lr():
        s = state["step"]
        f = (s + 1) / 201 if s < 200 else 1.0
        for gr, b in zip(opt.param_groups, base):
            gr["lr"] = b * f

    def fwd_bwd(tokens, labels):
        pred = model(tokens)
        loss = F.cross_entropy(pred.flatten(0, 1).float(), labels.flatten(0, 1))
        loss.backward()
        return loss

    def step_device(tokens, labels, timers=None):
        set_lr()
        loss = fwd_bwd(tokens, labels)
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0, foreach=True)
        if timers is not None:
            timers[0].record()
        opt.step()
        if timers is not None:
            timers[1].record()
        opt.zero_grad(set_to_none=True)
        state["step"] += 1
        return loss

    def step_e2e(tokens_host, labels_host):
        t = tokens_host.to("cuda", non_blocking=True)
        l = labels_host.to("cuda", non_blocking=True)
        return step_device(t, l).item()

    return step_device, step_e2e


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local)
    import datetime

    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    else:
        dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1,
                                timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    from torch.distributed.device_mesh import init_device_mesh

    W, K = args.warmup, args.steps
    lb, S = args.local_batch, args.seq_len
    tokens_per_step = lb * S * world

    if args.impl == "reference":
        if not os.path.isdir(os.path.join(REF_PATH, "ada_dion")):
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref not installed"}))
            return
        mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("dp_shard",))
        step_device, step_e2e = build_reference(args, world, mesh)
    else:
        step_device, step_e2e = build_ours(args, world)

    batches = make_batches(W + K, MODEL["vocab"], S, lb, rank, world, seed=2)
    dev_batches = [(t.cuda(), l.cuda()) for t, l in batches]

    # ---------------- warm-up
    for i in range(W):
        step_device(*dev_batches[i])
    barrier_sync()

    # ---------------- device-timed region
    try:
        import dion_b200.ops as _ops

        launches0 = _ops.ext().launch_count() if args.impl == "ours" else 0
    except Exception:
        launches0 = 0
    clocks = ClockSampler([local] if world == 1 else list(range(world)))
    if rank == 0:
        clocks.start()
    opt_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier_sync()
    start.record()
    last = None
    for i in range(K):
        last = step_device(*dev_batches[W + i], timers=opt_events[i])
    end.record()
    barrier_sync()
    clk = clocks.stop() if rank == 0 else None
    launches = (_ops.ext().launch_count() - launches0) if args.impl == "ours" else 0
    ms_total = max_over_ranks(start.elapsed_time(end))
    opt_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in opt_events) / K)
    ms_per_step = ms_total / K
    value = tokens_per_step * K / (ms_total / 1000.0)
    final_loss = float(last.item()) if last is not None else float("nan")

    # ---------------- end-to-end through the public per-step API
    e2e = None
    if not args.no_e2e:
        barrier_sync()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for i in range(K):
            step_e2e(*batches[(W + i) % len(batches)])
        e2.record()
        barrier_sync()
        e2e_ms = max_over_ranks(s2.elapsed_time(e2))
        h2d = sum(t.numel() * t.element_size() for t in batches[0])
        e2e = {"value": tokens_per_step * K / (e2e_ms / 1000.0), "unit": "tokens/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4, "ms_per_step": e2e_ms / K}

    if rank == 0:
        out = {
            "metric": "Llama tokens/sec + optimizer-step ms (max over ranks)",
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": K,
            "warmup": W,
            "ms_per_step": ms_per_step,
            "optimizer_step_ms": opt_ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic uniform tokens (seed 2), random init",
            "config": {"model": MODEL["name"], "global_batch": lb * world, "seq_len": S,
                       "parallelism": f"fsdp{world}", "optimizer": args.optimizer + "+adamw",
                       "l2": "working set >> 126 MB L2 (1.5B-param model, 32K-token steps)"},
            "final_loss": final_loss,
            "clocks": clk,
            "impl": args.impl,
        }
        if e2e is not None:
            out["e2e"] = e2e
        if args.impl == "ours":
            out["gpu_launches"] = launches
        print(json.dumps(out))
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
