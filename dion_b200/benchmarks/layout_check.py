"""Check every optimizer on every parallel layout, without GPUs.

    python -m dion_b200.benchmarks.layout_check --layouts 2x1x1x1,2x2x1x1,1x1x1x2,1x2x1x2,1x2x2x1 \\
        --optimizers all [--steps 3] [--json out.jsonl]

A layout is ``replicate x shard x tp x pp``; each runs as that many CPU
processes over gloo (the sharded, replicated, tensor- and pipeline-parallel
code paths of the trainer and optimizers, with the plain-PyTorch math) and
trains a small Llama for a few steps. One JSON line per (layout, optimizer):
``status`` ok (with the losses), unsupported (a combination the optimizer
declines up front, with its reason) or failed (with the last line of the
first failing rank's error). The
reference validates its configs the same way with torchtitan's fake backend
(ada_dion/scripts/run_local.sh); this check also covers the layout x
optimizer combinations. Exit status 1 when any combination fails.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import socket
import sys
import traceback
from typing import Dict, List, Sequence, Tuple

import torch

__all__ = ["OPTIMIZERS", "check", "main"]

OPTIMIZERS = ["Muon", "Dion", "Dion2", "AdaDionV2", "AdaDion", "AdaDionAnchor", "SDion", "GSDion", "AGDion",
              "QCDion", "AdamW"]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _train(name: str, layout: Tuple[int, int, int, int], steps: int) -> List[float]:
    from ..integration.hybrid_optimizer import HybridOptimizersContainer
    from ..integration.trainer import Trainer, TrainerConfig

    rep, shard, tp, pp = layout
    opt = HybridOptimizersContainer.Config(name=name, lr=0.02, init_rank=8, rank_min=4, rank_max=32, warmup_rank=16)
    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=4, vocab_size=512, max_seq_len=64), seq_len=32,
                        local_batch_size=4, steps=steps, warmup_steps=0, dp_replicate=rep, dp_shard=shard, tp=tp,
                        pp=pp, pp_microbatches=2, use_fsdp=rep * shard > 1 or tp > 1, optimizer=opt, seed=1)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    return [float(tr.train_step(*tr.data.next())) for _ in range(steps)]


def _rank_main(rank: int, world: int, port: int, name: str, layout, steps: int, q) -> None:
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        q.put((rank, "ok", _train(name, layout, steps)))
    except ValueError as e:  # a combination the optimizer declines up front (e.g. no TP path)
        q.put((rank, "unsupported", str(e)[:300]))
    except Exception:
        q.put((rank, "failed", traceback.format_exc().strip().splitlines()[-1][:300]))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def check(name: str, layout: Tuple[int, int, int, int], steps: int = 3) -> Dict:
    """Train ``name`` on ``layout`` with one gloo process per rank."""
    import torch.multiprocessing as mp

    world = layout[0] * layout[1] * layout[2] * layout[3]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, name, layout, steps, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, status, payload = q.get(timeout=600)
        results[r] = (status, payload)
    for p in procs:
        p.join(timeout=60)
    out = {"layout": "x".join(map(str, layout)), "optimizer": name}
    for status in ("failed", "unsupported"):
        ranks = sorted(r for r, (s, _) in results.items() if s == status)
        if ranks:
            out.update(status=status, rank=ranks[0], message=results[ranks[0]][1])
            return out
    out.update(status="ok", losses=results[0][1])
    return out


def _parse_layouts(spec: str) -> List[Tuple[int, int, int, int]]:
    out = []
    for item in spec.split(","):
        dims = tuple(int(v) for v in item.split("x"))
        if len(dims) != 4 or min(dims) < 1:
            raise SystemExit(f"layout {item!r}: expected replicate x shard x tp x pp, e.g. 2x2x1x1")
        out.append(dims)
    return out


def main(argv: Sequence[str] = None) -> List[Dict]:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--layouts", default="2x1x1x1,2x2x1x1,1x1x1x2,1x2x1x2,1x2x2x1")
    p.add_argument("--optimizers", default="all", help="comma-separated names, or 'all'")
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--json", default="", help="also append the JSON lines to this file")
    a = p.parse_args(argv)
    names = OPTIMIZERS if a.optimizers == "all" else a.optimizers.split(",")
    rows = []
    for layout in _parse_layouts(a.layouts):
        for name in names:
            row = check(name, layout, a.steps)
            rows.append(row)
            line = json.dumps(row)
            print(line, flush=True)
            if a.json:
                with open(a.json, "a") as f:
                    f.write(line + "\n")
    return rows


if __name__ == "__main__":
    rows = main()
    sys.exit(0 if all(r["status"] != "failed" for r in rows) else 1)
