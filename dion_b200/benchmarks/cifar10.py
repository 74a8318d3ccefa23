"""CIFAR-10 SmallViT benchmark: AdamW, Muon, Dion, Dion2, Dion-equivalent
AdaDionV2 and adaptive AdaDionV2, plus the reference's ablation presets
(benchmarks/cifar10_benchmark.py:137-225,517-637 of the reference), under
DDP (NCCL on GPUs, gloo on CPU).

Data: the torchvision CIFAR-10 files under ``--data-dir`` when present;
otherwise (no network here) a synthetic CIFAR-shaped set of the same size --
one random 32x32x3 template per class plus per-image noise, shifts and flips
-- which the output records as ``"data": "synthetic"``.

    python -m dion_b200.benchmarks.cifar10 --epochs 5 --optimizers adamw,muon,dion,adadion_v2
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m dion_b200.benchmarks.cifar10 ...
"""
from __future__ import annotations

import argparse
import json
import math
import os
import time
from collections import defaultdict
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

__all__ = ["SmallViT", "create_optimizer", "run_one", "synthetic_cifar", "ABLATION_MAP", "main"]

MEAN = torch.tensor([0.4914, 0.4822, 0.4465]).view(1, 3, 1, 1)
STD = torch.tensor([0.2470, 0.2435, 0.2616]).view(1, 3, 1, 1)


# ------------------------------------------------------------------ model
class _Block(nn.Module):
    def __init__(self, dim: int, heads: int):
        super().__init__()
        self.heads = heads
        self.norm1 = nn.LayerNorm(dim)
        self.qkv = nn.Linear(dim, 3 * dim)
        self.proj = nn.Linear(dim, dim)
        self.norm2 = nn.LayerNorm(dim)
        self.fc1 = nn.Linear(dim, 4 * dim)
        self.fc2 = nn.Linear(4 * dim, dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, n, d = x.shape
        q, k, v = self.qkv(self.norm1(x)).view(b, n, 3, self.heads, d // self.heads).permute(2, 0, 3, 1, 4)
        a = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(b, n, d)
        x = x + self.proj(a)
        return x + self.fc2(F.gelu(self.fc1(self.norm2(x))))


class SmallViT(nn.Module):
    """~4.8M-parameter ViT (4x4 patches, dim 256, depth 6, 8 heads); almost
    all weights are 2-D matrices, which is what Dion / Muon update."""

    def __init__(self, dim: int = 256, depth: int = 6, heads: int = 8, num_classes: int = 10, patch: int = 4):
        super().__init__()
        self.patch_embed = nn.Conv2d(3, dim, patch, patch)
        n = (32 // patch) ** 2
        self.cls_token = nn.Parameter(torch.randn(1, 1, dim) * 0.02)
        self.pos_embed = nn.Parameter(torch.randn(1, n + 1, dim) * 0.02)
        self.blocks = nn.Sequential(*[_Block(dim, heads) for _ in range(depth)])
        self.norm = nn.LayerNorm(dim)
        self.head = nn.Linear(dim, num_classes)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self.patch_embed(x).flatten(2).transpose(1, 2)
        x = torch.cat([self.cls_token.expand(x.size(0), -1, -1), x], dim=1) + self.pos_embed
        return self.head(self.norm(self.blocks(x)[:, 0]))


# ------------------------------------------------------------------ data
def synthetic_cifar(n_train: int = 50000, n_test: int = 10000, seed: int = 0):
    """Learnable CIFAR-shaped data: class template + noise (uint8 images, int64 labels)."""
    g = torch.Generator().manual_seed(seed)
    templates = torch.rand(10, 3, 32, 32, generator=g)
    templates = F.avg_pool2d(templates, 3, 1, 1)  # smooth, image-like

    def make(n, off):
        gg = torch.Generator().manual_seed(seed + off)
        y = torch.randint(0, 10, (n,), generator=gg)
        x = templates[y] * 0.6 + 0.4 * torch.rand(n, 3, 32, 32, generator=gg)
        return (x.clamp(0, 1) * 255).to(torch.uint8), y

    return make(n_train, 1), make(n_test, 2)


def _load_cifar(data_dir: Optional[str], seed: int):
    if data_dir and os.path.isdir(os.path.join(data_dir, "cifar-10-batches-py")):
        try:
            from torchvision import datasets

            tr = datasets.CIFAR10(data_dir, train=True, download=False)
            te = datasets.CIFAR10(data_dir, train=False, download=False)
            cv = lambda d: (torch.from_numpy(d.data).permute(0, 3, 1, 2).contiguous(),  # noqa: E731
                            torch.tensor(d.targets))
            return cv(tr), cv(te), "cifar10"
        except Exception:  # noqa: BLE001
            pass
    tr, te = synthetic_cifar(seed=seed)
    return tr, te, "synthetic"


def _augment(x: torch.Tensor, g: torch.Generator) -> torch.Tensor:
    """Random crop (pad 4) and horizontal flip on a uint8 batch, on its device."""
    b = x.size(0)
    xp = F.pad(x.float(), (4, 4, 4, 4))
    dx = torch.randint(0, 9, (b,), generator=g).tolist()
    dy = torch.randint(0, 9, (b,), generator=g).tolist()
    out = torch.stack([xp[i, :, dy[i]:dy[i] + 32, dx[i]:dx[i] + 32] for i in range(b)])
    flip = torch.rand(b, generator=g) < 0.5
    out[flip] = out[flip].flip(-1)
    return out


def _normalize(x: torch.Tensor) -> torch.Tensor:
    return (x.float() / 255.0 - MEAN.to(x.device)) / STD.to(x.device)


# ------------------------------------------------------------------ optimizers
def _split_params(model: nn.Module) -> Tuple[List[nn.Parameter], List[nn.Parameter]]:
    mat, scalar = [], []
    for p in model.parameters():
        (mat if p.ndim == 2 and min(p.shape) >= 2 else scalar).append(p)
    return mat, scalar


def create_optimizer(name: str, model: nn.Module, lr: float, wd: float, rank_fraction: float = 0.5,
                     adaptive: bool = False, ada_kwargs: Optional[dict] = None):
    """Optimizer by benchmark name; non-matrix parameters run AdamW at lr/10
    (the reference's factory, benchmarks/cifar10_benchmark.py:168-225)."""
    from .. import optim

    if name == "adamw":
        return torch.optim.AdamW(model.parameters(), lr=lr, weight_decay=wd)
    mat, scalar = _split_params(model)
    groups = [{"params": mat}]
    if scalar:
        groups.append({"params": scalar, "algorithm": "adamw", "lr": lr * 0.1, "weight_decay": wd,
                       "beta1": 0.9, "beta2": 0.95, "epsilon": 1e-8})
    if name == "muon":
        return optim.Muon(groups, lr=lr, mu=0.95, weight_decay=wd)
    if name == "dion":
        return optim.Dion(groups, lr=lr, rank_fraction=rank_fraction, weight_decay=wd)
    if name == "dion2":
        return optim.Dion2(groups, lr=lr, fraction=rank_fraction, ef_decay=0.95, weight_decay=wd)
    kw = dict(erank_ema_beta=0.5, rank_scale=1.5, rank_min=8, rank_quantize=4, rank_step_up=8, rank_step_down=4,
              adapt_step=1)
    kw.update(ada_kwargs or {})
    return optim.AdaDionV2(groups, lr=lr, mu=0.95, rank_fraction_max=0.7 if adaptive else rank_fraction,
                           weight_decay=wd, adaptive_rank=adaptive, init_rank_fraction=rank_fraction,
                           use_quality_control=adaptive, **kw)


# name -> (optimizer, adaptive, AdaDionV2 overrides, rank fraction)
ABLATION_MAP = {
    "ada_frozen": ("dion_equiv", True, {"adapt_step": 999999}, 0.5),
    "ada_beta99": ("dion_equiv", True, {"erank_ema_beta": 0.99}, 0.5),
    "ada_beta95": ("dion_equiv", True, {"erank_ema_beta": 0.95}, 0.5),
    "ada_conservative": ("dion_equiv", True, {"erank_ema_beta": 0.99, "rank_scale": 2.5, "rank_min": 32,
                                              "rank_step_down": 1, "rank_step_up": 2}, 0.5),
    "ada_rmin32": ("dion_equiv", True, {"rank_min": 32}, 0.5),
    "ada_scale2": ("dion_equiv", True, {"rank_scale": 2.0}, 0.5),
    "dion_r07": ("dion_equiv", False, None, 0.7),
    "dion_r03": ("dion_equiv", False, None, 0.3),
}


# ------------------------------------------------------------------ training
@torch.no_grad()
def evaluate(model: nn.Module, x: torch.Tensor, y: torch.Tensor, bs: int = 1000) -> Tuple[float, float]:
    model.eval()
    loss = correct = 0.0
    for i in range(0, x.size(0), bs):
        lo = model(_normalize(x[i:i + bs]))
        loss += float(F.cross_entropy(lo, y[i:i + bs], reduction="sum"))
        correct += float((lo.argmax(1) == y[i:i + bs]).sum())
    model.train()
    return loss / x.size(0), correct / x.size(0)


def run_one(cfg: dict, data, device: torch.device, rank: int = 0, world: int = 1) -> Dict[str, list]:
    (xtr, ytr), (xte, yte) = data
    torch.manual_seed(cfg["seed"])
    model = SmallViT().to(device)
    if world > 1:
        model = nn.parallel.DistributedDataParallel(model, device_ids=[device.index] if device.type == "cuda" else None)
    core = model.module if world > 1 else model
    opt = create_optimizer(cfg["optimizer"], core, cfg["lr"], cfg["weight_decay"], cfg.get("rank_fraction", 0.5),
                           cfg.get("adaptive_rank", False), cfg.get("ada_kwargs"))
    bs = cfg["batch_size"]
    per_rank = xtr.size(0) // world
    steps_per_epoch = per_rank // bs
    total = cfg["epochs"] * steps_per_epoch
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=max(1, total))
    g = torch.Generator().manual_seed(cfg["seed"] + 17 * rank)
    xtr_d, ytr_d = xtr.to(device), ytr.to(device)
    xte_d, yte_d = xte.to(device), yte.to(device)
    log: Dict[str, list] = defaultdict(list)
    step, t0 = 0, time.time()
    for epoch in range(cfg["epochs"]):
        perm = torch.randperm(xtr.size(0), generator=torch.Generator().manual_seed(cfg["seed"] + epoch))
        mine = perm[rank * per_rank:(rank + 1) * per_rank]
        ep_loss = 0.0
        for it in range(steps_per_epoch):
            idx = mine[it * bs:(it + 1) * bs].to(device)
            xb = _normalize(_augment(xtr_d[idx], g).to(device)) if cfg.get("augment", True) else _normalize(xtr_d[idx])
            loss = F.cross_entropy(model(xb), ytr_d[idx])
            loss.backward()
            gnorm = float(torch.nn.utils.clip_grad_norm_(model.parameters(), max_norm=1e9))
            opt.step()
            opt.zero_grad(set_to_none=True)
            sched.step()
            step += 1
            ep_loss += float(loss.detach())
            if step % cfg["log_freq"] == 0 and rank == 0:
                row = {"step": step, "epoch": epoch, "train_loss": float(loss.detach()), "lr": sched.get_last_lr()[0],
                       "grad_norm": gnorm, "elapsed": time.time() - t0,
                       "throughput": step * bs * world / (time.time() - t0),
                       "mem_mb": torch.cuda.max_memory_allocated(device) / 1e6 if device.type == "cuda" else 0.0}
                for getter, key in (("get_rank", "rank"), ("get_effective_rank", "erank"), ("get_aerr", "aerr")):
                    if hasattr(opt, getter):
                        vals = list(getattr(opt, getter)().values())
                        if vals:
                            row[f"{key}_mean"] = sum(vals) / len(vals)
                            if key == "rank":
                                row["rank_min"], row["rank_max"] = min(vals), max(vals)
                for k, v in row.items():
                    log[k].append(v)
        val_loss, val_acc = evaluate(core, xte_d, yte_d)
        if rank == 0:
            for k, v in {"epoch": epoch, "step": step, "train_loss_epoch": ep_loss / max(1, steps_per_epoch),
                         "val_loss": val_loss, "val_acc": val_acc, "val_ppl": math.exp(min(val_loss, 20)),
                         "elapsed": time.time() - t0}.items():
                log[f"eval/{k}"].append(v)
            print(f"  [{cfg['name']}] ep {epoch + 1}/{cfg['epochs']} train={ep_loss / max(1, steps_per_epoch):.4f} "
                  f"val={val_loss:.4f} acc={val_acc:.4f} {time.time() - t0:.0f}s", flush=True)
    return dict(log)


def _plots(all_logs: Dict[str, dict], outdir: str) -> None:
    from ..utils.svgplot import Figure

    fig = Figure(ncols=3, title="CIFAR-10 SmallViT")
    for name, log in all_logs.items():
        if log.get("step"):
            fig.axes[0].line(log["step"], log["train_loss"], label=name)
        if log.get("eval/epoch"):
            fig.axes[1].line([e + 1 for e in log["eval/epoch"]], log["eval/val_acc"], label=name, markers=True)
        if log.get("rank_mean"):
            fig.axes[2].line(log["step"], log["rank_mean"], label=name)
    fig.axes[0].set(title="train loss", xlabel="step")
    fig.axes[1].set(title="val accuracy", xlabel="epoch")
    fig.axes[2].set(title="mean Dion rank", xlabel="step")
    fig.save(os.path.join(outdir, "cifar10.svg"))


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--epochs", type=int, default=50)
    p.add_argument("--batch-size", type=int, default=128)
    p.add_argument("--lr", type=float, default=0.1, help="AdamW learning rate (matrix optimizers use 0.02)")
    p.add_argument("--wd", type=float, default=5e-4)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--log-freq", type=int, default=20)
    p.add_argument("--outdir", default="cifar10_results")
    p.add_argument("--data-dir", default="./data")
    p.add_argument("--optimizers", default="adamw,muon,dion,dion2,dion_equiv,adadion_v2")
    p.add_argument("--train-size", type=int, default=None, help="use the first N training images")
    p.add_argument("--no-augment", action="store_true")
    a = p.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cuda = torch.cuda.is_available()
    device = torch.device("cuda", local) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl" if cuda else "gloo")
    (xtr, ytr), (xte, yte), src = _load_cifar(a.data_dir, a.seed)
    if a.train_size:
        xtr, ytr = xtr[:a.train_size], ytr[:a.train_size]
        xte, yte = xte[:max(1000, a.train_size // 5)], yte[:max(1000, a.train_size // 5)]
    lr_map = {"adamw": a.lr}
    all_logs = {}
    for name in [o.strip() for o in a.optimizers.split(",") if o.strip()]:
        if name in ABLATION_MAP:
            base, adaptive, ada_kw, rf = ABLATION_MAP[name]
        else:
            base, adaptive, ada_kw, rf = name, name == "adadion_v2", None, 0.5
        cfg = {"name": name, "optimizer": base, "epochs": a.epochs, "batch_size": a.batch_size,
               "lr": lr_map.get(name, 0.02), "weight_decay": a.wd, "seed": a.seed, "log_freq": a.log_freq,
               "rank_fraction": rf, "adaptive_rank": adaptive, "ada_kwargs": ada_kw, "augment": not a.no_augment}
        if rank == 0:
            print(f"--- {name} (lr={cfg['lr']}, data={src}) ---", flush=True)
        all_logs[name] = run_one(cfg, ((xtr, ytr), (xte, yte)), device, rank, world)
    if rank == 0:
        os.makedirs(a.outdir, exist_ok=True)
        summary = {n: {"final_val_acc": l.get("eval/val_acc", [float("nan")])[-1],
                       "final_val_loss": l.get("eval/val_loss", [float("nan")])[-1]} for n, l in all_logs.items()}
        with open(os.path.join(a.outdir, "results.json"), "w") as f:
            json.dump({"data": src, "world_size": world, "summary": summary, "logs": all_logs}, f)
        _plots(all_logs, a.outdir)
        print(json.dumps({"data": src, "summary": summary}), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return all_logs


if __name__ == "__main__":
    main()
