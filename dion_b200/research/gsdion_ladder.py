"""GSDion ablation ladder: starting from plain Dion, switch on one GSDion
mechanism at a time (rank normalisation with sqrt(r) lr compensation, RMS
matching, bounded centred scalar, trust region, residual-driven rank), same
seed and data for every rung (ada_dion/scripts/run_gsdion_comparison.py:43-97).

    python -m dion_b200.research.gsdion_ladder --steps 500 [--configs 1_dion_baseline,7_full_gsdion]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import time
from typing import Dict, List

import torch
import torch.nn.functional as F

from ..optim import GSDion
from .common import MLP, batches, evaluate, load_fmnist

_OFF = dict(rank_normalize=False, use_adaptive_scalar=False, use_rms_matching=False, use_trust_region=False,
            use_residual_rank=False, use_pre_balance=False, use_anchor=False)


def _on(**kw):
    d = dict(_OFF)
    d.update(kw)
    return d


CONFIGS: Dict[str, dict] = {
    "1_dion_baseline": _on(),
    "2_ranknorm_lrcomp": _on(rank_normalize=True),
    "3_ranknorm_rms": _on(rank_normalize=True, use_rms_matching=True),
    "4_ranknorm_scalar": _on(rank_normalize=True, use_adaptive_scalar=True),
    "5_ranknorm_rms_scalar": _on(rank_normalize=True, use_adaptive_scalar=True, use_rms_matching=True),
    "6_ranknorm_rms_scalar_tr": _on(rank_normalize=True, use_adaptive_scalar=True, use_rms_matching=True,
                                    use_trust_region=True),
    "7_full_gsdion": _on(rank_normalize=True, use_adaptive_scalar=True, use_rms_matching=True, use_trust_region=True,
                         use_residual_rank=True),
}
# rung 2 compensates the 1/sqrt(r) of rank normalisation in the learning rate
LR_COMPENSATED = {"2_ranknorm_lrcomp"}


def run_single(name: str, data, steps: int, lr: float, init_rank: int, hidden: int, bs: int, eval_freq: int,
               seed: int) -> dict:
    (xtr, ytr), (xte, yte) = data
    torch.manual_seed(seed)
    model = MLP(hidden)
    run_lr = lr * math.sqrt(init_rank) if name in LR_COMPENSATED else lr
    opt = GSDion(model.parameters(), lr=run_lr, init_rank=init_rank, rank_max=max(init_rank, 256),
                 **CONFIGS[name])
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=steps)
    it = batches(xtr, ytr, bs, seed)
    rows: List[dict] = []
    t0 = time.time()
    for step in range(1, steps + 1):
        x, y = next(it)
        loss = F.cross_entropy(model(x), y)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        sched.step()
        if step % eval_freq == 0 or step == steps:
            vl, va, vp = evaluate(model, xte, yte)
            row = {"step": step, "train_loss": float(loss.detach()), "val_loss": vl, "val_acc": va, "val_ppl": vp,
                   "time_s": time.time() - t0}
            ranks = list(opt.get_rank().values()) if hasattr(opt, "get_rank") else []
            if ranks:
                row["rank_mean"] = sum(ranks) / len(ranks)
            rows.append(row)
    return {"name": name, "lr": run_lr, "rows": rows, "final": rows[-1]}


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--steps", type=int, default=500)
    p.add_argument("--lr", type=float, default=0.02)
    p.add_argument("--init-rank", type=int, default=64)
    p.add_argument("--hidden", type=int, default=1024)
    p.add_argument("--batch-size", type=int, default=256)
    p.add_argument("--eval-freq", type=int, default=50)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--outdir", default="gsdion_results")
    p.add_argument("--data-dir", default="./data")
    p.add_argument("--configs", default="all")
    a = p.parse_args(argv)
    names = list(CONFIGS) if a.configs == "all" else [n.strip() for n in a.configs.split(",")]
    tr, te, src = load_fmnist(a.data_dir, a.seed)
    results = {}
    for n in names:
        r = run_single(n, (tr, te), a.steps, a.lr, a.init_rank, a.hidden, a.batch_size, a.eval_freq, a.seed)
        results[n] = r
        f = r["final"]
        print(f"{n:<28s} lr={r['lr']:.4f} val_loss={f['val_loss']:.4f} val_acc={f['val_acc']:.4f}", flush=True)
    os.makedirs(a.outdir, exist_ok=True)
    with open(os.path.join(a.outdir, "gsdion_ladder.json"), "w") as fh:
        json.dump({"data": src, "results": results}, fh)
    return results


if __name__ == "__main__":
    main()
