"""Whole pipeline on one machine, with measured data only: every optimizer
trains the small Llama through the package's trainer, the optimizer
diagnostics are recorded each step, tier A runs, the sweep grid is
validated, and the full plot set is written (the reference's
run_full_pipeline_local.py draws its comparison curves from synthetic
numbers; here every curve is a real run).

    python -m dion_b200.research.pipeline_local --steps 50 --outdir pipeline_out [--model tiny]
"""
from __future__ import annotations

import argparse
import json
import os
import time
from typing import Dict

import torch

from ..benchmarks import plots, sweep, tiers
from ..integration.hybrid_optimizer import HybridOptimizersContainer
from ..integration.trainer import Trainer, TrainerConfig

OPTIMIZERS = {"adamw": ("AdamW", 3e-3), "muon": ("Muon", 0.02), "dion": ("Dion", 0.02), "dion2": ("Dion2", 0.02),
              "adadion": ("AdaDion", 0.02), "adadion_v2": ("AdaDionV2", 0.02)}


def _mean(d) -> float:
    v = [float(x) for x in d.values()] if isinstance(d, dict) else []
    return sum(v) / len(v) if v else float("nan")


def run_optimizer(key: str, steps: int, model: str, seq: int, batch: int, seed: int) -> Dict[str, list]:
    name, lr = OPTIMIZERS[key]
    ocfg = HybridOptimizersContainer.Config(name=name, lr=lr, scalar_lr=3e-3, init_rank=16, rank_min=4,
                                            rank_max=64)
    tc = TrainerConfig(model=model, seq_len=seq, local_batch_size=batch, steps=steps, warmup_steps=max(1, steps // 10),
                       optimizer=ocfg, seed=seed, use_fsdp=False)
    tr = Trainer(tc)
    out: Dict[str, list] = {k: [] for k in ("step", "tokens", "train_loss", "time_s", "tokens_per_sec", "rank_mean",
                                            "residual_norm_mean", "aerr_mean", "erank_mean")}
    t0 = time.perf_counter()
    tok = seq * batch
    for s in range(1, steps + 1):
        t, l = tr.data.next()
        ts = time.perf_counter()
        loss = float(tr.train_step(t, l))
        if tr.device.type == "cuda":
            torch.cuda.synchronize()
        dt = time.perf_counter() - ts
        out["step"].append(s)
        out["tokens"].append(s * tok)
        out["train_loss"].append(loss)
        out["time_s"].append(time.perf_counter() - t0)
        out["tokens_per_sec"].append(tok / dt)
        opt = tr.optimizers.optimizers[0]
        out["rank_mean"].append(_mean(opt.get_rank()) if hasattr(opt, "get_rank") else float("nan"))
        out["erank_mean"].append(_mean(opt.get_effective_rank()) if hasattr(opt, "get_effective_rank") else float("nan"))
        out["aerr_mean"].append(_mean(opt.get_aerr()) if hasattr(opt, "get_aerr") else float("nan"))
        ms = [float(st["momentum"].float().norm()) for st in opt.state.values() if isinstance(st, dict)
              and "momentum" in st and getattr(st["momentum"], "ndim", 0) == 2]
        out["residual_norm_mean"].append(sum(ms) / len(ms) if ms else float("nan"))
    return out


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--model", default="tiny")
    p.add_argument("--seq-len", type=int, default=128)
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--optimizers", default=",".join(OPTIMIZERS))
    p.add_argument("--outdir", default="pipeline_out")
    a = p.parse_args(argv)
    os.makedirs(a.outdir, exist_ok=True)
    runs = {}
    for k in [x.strip() for x in a.optimizers.split(",") if x.strip()]:
        r = run_optimizer(k, a.steps, a.model, a.seq_len, a.batch, a.seed)
        runs[k] = r
        print(f"{k:<11s} loss {r['train_loss'][0]:.3f} -> {r['train_loss'][-1]:.3f}  "
              f"median tps {sorted(r['tokens_per_sec'])[len(r['tokens_per_sec']) // 2]:,.0f}", flush=True)
    tier_a = tiers.run_tier_a("cuda" if torch.cuda.is_available() else "cpu")
    grid = sweep.generate_sweep_configs()
    curves = {k: {"tokens": v["tokens"], "val_loss": v["train_loss"], "time_s": v["time_s"], "step": v["step"],
                  "tokens_per_sec": v["tokens_per_sec"]} for k, v in runs.items()}
    dion_data = ({"step": runs["dion"]["step"], "rank_mean": runs["dion"]["rank_mean"],
                  "residual_norm_mean": runs["dion"]["residual_norm_mean"]} if "dion" in runs else None)
    ada = runs.get("adadion_v2") or runs.get("adadion")
    ada_data = ({"step": ada["step"], "rank_mean": ada["rank_mean"], "erank_mean": ada["erank_mean"],
                 "aerr_mean": ada["aerr_mean"]} if ada else None)
    written = plots.save_all_plots(os.path.join(a.outdir, "plots"), runs=curves, dion_data=dion_data,
                                   adadion_data=ada_data)
    summary = {"runs": runs, "tier_a": tier_a, "sweep_runs": len(grid), "plots": written,
               "note": "every curve is a measured run of this package on this machine"}
    with open(os.path.join(a.outdir, "pipeline.json"), "w") as f:
        json.dump(summary, f)
    print(json.dumps({"tier_a_pass": all(v["pass"] for v in tier_a.values()), "sweep_runs": len(grid),
                      "plots": len(written)}))
    return summary


if __name__ == "__main__":
    main()
