"""Seed confirmation: plain Dion vs rank-normalised Dion (lr x sqrt(r)) over
several seeds on the MLP task, with the final weight-direction cosine between
the two runs of each seed (ada_dion/scripts/run_seed_confirmation.py).

    python -m dion_b200.research.seed_confirmation --steps 500 --seeds 42,123,7,2024,314
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics

import torch
import torch.nn.functional as F

from ..optim import GSDion
from .common import MLP, batches, evaluate, load_fmnist, weight_cosines
from .gsdion_ladder import CONFIGS


def _train(seed, data, steps, lr, init_rank, hidden, bs, kw):
    (xtr, ytr), (xte, yte) = data
    torch.manual_seed(seed)
    model = MLP(hidden)
    opt = GSDion(model.parameters(), lr=lr, init_rank=init_rank, rank_max=max(256, init_rank), **kw)
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=steps)
    it = batches(xtr, ytr, bs, seed)
    for _ in range(steps):
        x, y = next(it)
        F.cross_entropy(model(x), y).backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        sched.step()
    vl, va, _ = evaluate(model, xte, yte)
    return model, vl, va


def run_pair(seed, data, steps=500, init_rank=64, lr=0.02, hidden=1024, bs=256):
    d_model, d_vl, d_va = _train(seed, data, steps, lr, init_rank, hidden, bs, CONFIGS["1_dion_baseline"])
    n_model, n_vl, n_va = _train(seed, data, steps, lr * math.sqrt(init_rank), init_rank, hidden, bs,
                                 CONFIGS["2_ranknorm_lrcomp"])
    cos = weight_cosines(d_model, n_model)
    return {"seed": seed, "dion_val_loss": d_vl, "dion_val_acc": d_va, "normdion_val_loss": n_vl,
            "normdion_val_acc": n_va, **{f"cosine_{k.split('.')[0]}": v for k, v in cos.items()},
            "cosine_mean": sum(cos.values()) / len(cos)}


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--steps", type=int, default=500)
    p.add_argument("--seeds", default="42,123,7,2024,314")
    p.add_argument("--init-rank", type=int, default=64)
    p.add_argument("--lr", type=float, default=0.02)
    p.add_argument("--hidden", type=int, default=1024)
    p.add_argument("--batch-size", type=int, default=256)
    p.add_argument("--data-dir", default="./data")
    p.add_argument("--outdir", default="seed_confirmation")
    a = p.parse_args(argv)
    tr, te, src = load_fmnist(a.data_dir, 0)
    rows = []
    for s in [int(x) for x in a.seeds.split(",")]:
        r = run_pair(s, (tr, te), a.steps, a.init_rank, a.lr, a.hidden, a.batch_size)
        rows.append(r)
        print(f"seed {s}: dion acc={r['dion_val_acc']:.4f} normdion acc={r['normdion_val_acc']:.4f} "
              f"cos={r['cosine_mean']:.4f}", flush=True)
    def ms(k):
        v = [r[k] for r in rows]
        return statistics.mean(v), (statistics.stdev(v) if len(v) > 1 else 0.0)
    summary = {k: ms(k) for k in ("dion_val_acc", "normdion_val_acc", "dion_val_loss", "normdion_val_loss",
                                  "cosine_mean")}
    print(json.dumps({"data": src, "summary": summary}))
    os.makedirs(a.outdir, exist_ok=True)
    with open(os.path.join(a.outdir, "seed_confirmation.json"), "w") as fh:
        json.dump({"data": src, "rows": rows, "summary": summary}, fh)
    return rows, summary


if __name__ == "__main__":
    main()
