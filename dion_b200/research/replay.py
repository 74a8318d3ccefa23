"""Trace-and-replay study of Dion update rules
(ada_dion/scripts/part_a_replay.py, part_a_collect.sh).

Phase 1 (``collect``): train with Dion and, every ``--freq`` steps, save a
snapshot ``{step, loss, layers: [{name, grad, M, shape}]}`` of every matrix
parameter's gradient and Dion momentum (``torch.save``, one file per step).
The model is the MLP task by default or any registered trainer config
(``--config llama3_debug_dion``).

Phase 2 (``replay``): on every snapshot, layer and rank, apply four update
rules to the same (M, G) from the same initial basis and record the update's
Frobenius norm and RMS, the scalars s_t / c_t, the cosine to the Dion update,
<M, update> and the latency:

  dion             D = P Q^T                      (one power step, Cholesky QR)
  normdion         D / sqrt(r), lr x sqrt(r)
  normdion_cs      + centred log-RMS scalar s_t = clip(exp(-rho (log rms(G) - EMA)), 1/gamma, gamma)
  normdion_cs_rms  + RMS matching c_t = rms(M) / rms(D)

    python -m dion_b200.research.replay collect --steps 200 --freq 50 --snapshot-dir snaps
    python -m dion_b200.research.replay replay --snapshot-dir snaps --ranks 16,32 --outdir replay_results
"""
from __future__ import annotations

import argparse
import json
import math
import os
import time
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor

__all__ = ["dion_direction", "replay_step", "collect", "replay", "VARIANTS"]

VARIANTS = ("dion", "normdion", "normdion_cs", "normdion_cs_rms")


def _rms(t: Tensor) -> float:
    return float(t.float().pow(2).mean().sqrt().clamp_min(1e-12))


def _orthonormal_columns(P: Tensor) -> Tensor:
    """Cholesky QR of P (n x r, fp32); Householder QR when the Gram is singular."""
    G = P.T @ P
    G.diagonal().add_(1e-6)
    L, info = torch.linalg.cholesky_ex(G)
    if int(info) == 0:
        return torch.linalg.solve_triangular(L, P.T, upper=False).T
    return torch.linalg.qr(P)[0]


def dion_direction(B: Tensor, Q: Tensor, r: int) -> Tuple[Tensor, Tensor, Tensor]:
    """One power step on B (m x n) from basis Q: returns (D = P Q_new^T, Q_new, P R^T)."""
    m, n = B.shape
    tall = m > n
    A = (B.T if tall else B).float()        # rows >= cols after orientation
    P = _orthonormal_columns(A @ Q[:, :r].float())
    R = A.T @ P
    Qn = R / R.norm(dim=0, keepdim=True).clamp_min(1e-12)
    D, approx = P @ Qn.T, P @ R.T
    if tall:
        D, approx = D.T, approx.T
    return D, Qn, approx


def replay_step(M: Tensor, G: Tensor, Q0: Tensor, r: int, variant: str, state: dict, mu: float = 0.95,
                lr: float = 0.02, rho: float = 0.3, gamma: float = 1.2, beta: float = 0.99) -> dict:
    t0 = time.perf_counter()
    B = mu * M.float() + G.float()
    D_raw, _, _ = dion_direction(B, Q0, r)
    m, n = M.shape
    shape_scale = math.sqrt(min(m, n) / max(m, n))
    D, eff_lr = (D_raw / math.sqrt(r), lr * math.sqrt(r)) if variant != "dion" else (D_raw, lr)
    s_t = 1.0
    if variant in ("normdion_cs", "normdion_cs_rms"):
        lg = math.log(_rms(G))
        state["log_ema"] = lg if "log_ema" not in state else beta * state["log_ema"] + (1 - beta) * lg
        s_t = min(gamma, max(1.0 / gamma, math.exp(-rho * (lg - state["log_ema"]))))
    c_t = _rms(M) / _rms(D) if variant == "normdion_cs_rms" else 1.0
    update = D * (eff_lr * shape_scale * c_t * s_t)
    return {"update": update, "update_fro": float(update.norm()), "update_rms": _rms(update), "s_t": s_t,
            "c_t": c_t, "cs_product": c_t * s_t, "latency_ms": (time.perf_counter() - t0) * 1e3}


# ------------------------------------------------------------------ phase 1
def collect(steps: int, freq: int, snapshot_dir: str, config: Optional[str] = None, seed: int = 0,
            data_dir: str = "./data") -> List[str]:
    from ..optim import Dion

    os.makedirs(snapshot_dir, exist_ok=True)
    written = []
    if config:
        from ..train import _load_config, trainer_config_from_job
        from ..integration.trainer import Trainer

        tc = trainer_config_from_job(_load_config(None, config))
        tc.steps = steps
        tr = Trainer(tc)
        model, opt = tr.model, tr.optimizers

        def next_loss():
            t, l = tr.data.next()
            return tr.model.loss(t.to(tr.device), l.to(tr.device))

        inner = [o for o in tr.optimizers if isinstance(o, Dion)]
        dion_opt = inner[0] if inner else None
    else:
        from .common import MLP, batches, load_fmnist

        (xtr, ytr), _, _ = load_fmnist(data_dir, seed, n_train=20000, n_test=1000)
        torch.manual_seed(seed)
        model = MLP(512)
        opt = dion_opt = Dion(model.parameters(), lr=0.02, rank_fraction=0.25)
        it = batches(xtr, ytr, 256, seed)

        def next_loss():
            x, y = next(it)
            return F.cross_entropy(model(x), y)

    for step in range(1, steps + 1):
        loss = next_loss()
        loss.backward()
        if step % freq == 0 and dion_opt is not None:
            layers = []
            for name, p in model.named_parameters():
                st = dion_opt.state.get(p, {})
                if p.ndim != 2 or p.grad is None or "momentum" not in st:
                    continue
                full = lambda t: t.full_tensor() if hasattr(t, "full_tensor") else t  # noqa: E731
                layers.append({"name": name, "grad": full(p.grad).detach().float().cpu(),
                               "M": full(st["momentum"]).detach().float().cpu(), "shape": tuple(p.shape)})
            path = os.path.join(snapshot_dir, f"snap_{step:06d}.pt")
            torch.save({"step": step, "loss": float(loss.detach()), "layers": layers}, path)
            written.append(path)
        opt.step()
        opt.zero_grad(set_to_none=True)
    return written


# ------------------------------------------------------------------ phase 2
def replay(snapshot_dir: str, ranks: List[int], outdir: str, lr: float = 0.02, mu: float = 0.95) -> List[dict]:
    files = sorted(f for f in os.listdir(snapshot_dir) if f.endswith(".pt"))
    rows: List[dict] = []
    states: Dict[Tuple[str, str, int], dict] = {}
    for fname in files:
        snap = torch.load(os.path.join(snapshot_dir, fname), weights_only=False)
        for r in ranks:
            for layer in snap["layers"]:
                M, G, name = layer["M"], layer["grad"], layer["name"]
                m, n = M.shape
                if r > min(m, n):
                    continue
                # same initial basis for every rule: rows = the right dimension after orientation
                g = torch.Generator().manual_seed(0x4753 + n * 1000 + r)
                Q0 = F.normalize(torch.randn(m if m > n else n, r, generator=g), dim=0)
                row = {"step": snap["step"], "loss": snap["loss"], "layer": name, "rank": r, "shape": f"{m}x{n}",
                       "grad_rms": _rms(G), "M_rms": _rms(M)}
                ref = None
                for v in VARIANTS:
                    res = replay_step(M, G, Q0, r, v, states.setdefault((v, name, r), {}), mu=mu, lr=lr)
                    if v == "dion":
                        ref = res["update"]
                    cos = float(F.cosine_similarity(res["update"].flatten(), ref.flatten(), dim=0))
                    row.update({f"{v}/update_fro": res["update_fro"], f"{v}/update_rms": res["update_rms"],
                                f"{v}/s_t": res["s_t"], f"{v}/c_t": res["c_t"], f"{v}/cs": res["cs_product"],
                                f"{v}/cos_to_dion": cos,
                                f"{v}/scalar_product": float((M.float() * res["update"]).sum()),
                                f"{v}/latency_ms": res["latency_ms"]})
                row["rms_ratio_new_vs_dion"] = row["normdion_cs_rms/update_rms"] / (row["dion/update_rms"] + 1e-12)
                rows.append(row)
    os.makedirs(outdir, exist_ok=True)
    with open(os.path.join(outdir, "replay_analysis.json"), "w") as f:
        json.dump(rows, f, indent=1)
    for r in ranks:
        sel = [x for x in rows if x["rank"] == r]
        if not sel:
            continue
        print(f"rank {r}:")
        for v in VARIANTS:
            mean = lambda k: sum(x[f"{v}/{k}"] for x in sel) / len(sel)  # noqa: E731
            print(f"  {v:<18s} cos={mean('cos_to_dion'):.4f} s_t={mean('s_t'):.4f} "
                  f"update_rms={mean('update_rms'):.3e}")
    return rows


def main(argv=None):
    p = argparse.ArgumentParser()
    sub = p.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("collect")
    c.add_argument("--steps", type=int, default=500)
    c.add_argument("--freq", type=int, default=50)
    c.add_argument("--snapshot-dir", default="replay_snapshots")
    c.add_argument("--config", default=None)
    c.add_argument("--seed", type=int, default=0)
    c.add_argument("--data-dir", default="./data")
    r = sub.add_parser("replay")
    r.add_argument("--snapshot-dir", default="replay_snapshots")
    r.add_argument("--outdir", default="replay_results")
    r.add_argument("--ranks", default="64,128")
    r.add_argument("--lr", type=float, default=0.02)
    r.add_argument("--mu", type=float, default=0.95)
    a = p.parse_args(argv)
    if a.cmd == "collect":
        for w in collect(a.steps, a.freq, a.snapshot_dir, a.config, a.seed, a.data_dir):
            print(w)
    else:
        replay(a.snapshot_dir, [int(x) for x in a.ranks.split(",")], a.outdir, a.lr, a.mu)


if __name__ == "__main__":
    main()
