"""Per-step optimizer telemetry written as JSON lines (and optionally to
TensorBoard / W&B writers the caller owns).

Same interface and record layout as the reference's collector
(ada_dion/benchmarks/metrics_collector.py:22-137): one record per
``collect(step)`` with ``step``, ``timestamp``, ``opt_<i>/type`` and, for
each optimizer, its diagnostics (rank, effective rank, approximation error,
anchor drift, tail ratio, per-variant diagnostics) plus ``grad_norm`` and
``param_norm``. Differences: diagnostics are discovered by duck typing, so
any optimizer of this package reports what it has; the norms come from one
batched device reduction and one device->host copy per optimizer instead of
two ``.item()`` calls per parameter.
"""
from __future__ import annotations

import json
import os
import time
from collections import defaultdict
from typing import Any, Dict, List, Optional

import torch

from .. import ops

__all__ = ["OptimizerMetricsCollector"]

_GETTERS = (
    ("rank", "get_rank"),
    ("erank", "get_effective_rank"),
    ("aerr", "get_aerr"),
    ("anchor_drift", "get_anchor_drift"),
    ("tail_ratio", "get_tail_ratio"),
    ("diag", "get_diagnostics"),
)


def _local(t: torch.Tensor) -> torch.Tensor:
    return t.to_local() if hasattr(t, "to_local") else t


class OptimizerMetricsCollector:
    def __init__(self, matrix_optimizers, output_dir: str = "./metrics", tb_writer=None, wandb_run=None,
                 filename: str = "optimizer_metrics.jsonl"):
        if hasattr(matrix_optimizers, "get_optimizers"):
            matrix_optimizers = matrix_optimizers.get_optimizers()
        if not isinstance(matrix_optimizers, (list, tuple)):
            matrix_optimizers = [matrix_optimizers]
        self.matrix_optimizers = list(matrix_optimizers)
        self.output_dir = output_dir
        self.tb_writer = tb_writer
        self.wandb_run = wandb_run
        self._history: Dict[str, List[Any]] = defaultdict(list)
        os.makedirs(output_dir, exist_ok=True)
        self._jsonl_path = os.path.join(output_dir, filename)
        self._jsonl_file = open(self._jsonl_path, "a")

    @staticmethod
    def _norms(opt) -> Optional[Dict[str, float]]:
        """Norms of this rank's parameter shards (and of their gradients while
        they exist: a trainer that clears gradients before collecting gets the
        parameter norm only)."""
        grads, params = [], []
        for g in opt.param_groups:
            for p in g["params"]:
                params.append(_local(p).detach())
                if p.grad is not None:
                    grads.append(_local(p.grad).detach())
        if not params:
            return None

        def sumsq(ts):
            if not ts:
                return torch.zeros((), device=params[0].device)
            if ts[0].is_cuda:
                return ops.multi_sumsq([t.contiguous() for t in ts]).sum()
            return torch.stack([t.float().square().sum() for t in ts]).sum()

        both = torch.stack([sumsq(grads), sumsq(params)]).cpu().tolist()
        out = {"param_norm": both[1] ** 0.5}
        if grads:
            out["grad_norm"] = both[0] ** 0.5
        return out

    def collect(self, step: int, **extra: Any) -> Dict[str, Any]:
        metrics: Dict[str, Any] = {"step": step, "timestamp": time.time()}
        metrics.update(extra)
        for i, opt in enumerate(self.matrix_optimizers):
            prefix = f"opt_{i}"
            metrics[f"{prefix}/type"] = type(opt).__name__
            for label, getter in _GETTERS:
                fn = getattr(opt, getter, None)
                if fn is None:
                    continue
                try:
                    vals = fn()
                except (RuntimeError, KeyError, ValueError):
                    continue
                for name, val in (vals or {}).items():
                    metrics[f"{prefix}/{label}/{name}"] = val
            n = self._norms(opt)
            for k, v in (n or {}).items():
                metrics[f"{prefix}/{k}"] = v
        for k, v in metrics.items():
            if k not in ("step", "timestamp"):
                self._history[k].append(v)
        self._jsonl_file.write(json.dumps(metrics, default=str) + "\n")
        self._jsonl_file.flush()
        scalars = {k: v for k, v in metrics.items()
                   if k not in ("step", "timestamp") and isinstance(v, (int, float)) and not isinstance(v, bool)}
        if self.tb_writer is not None:
            for k, v in scalars.items():
                self.tb_writer.add_scalar(f"optimizer/{k}", v, step)
        if self.wandb_run is not None:
            self.wandb_run.log({f"optimizer/{k}": v for k, v in scalars.items()}, step=step)
        return metrics

    def get_history(self) -> Dict[str, List[Any]]:
        return dict(self._history)

    def close(self) -> None:
        if self._jsonl_file:
            self._jsonl_file.close()
            self._jsonl_file = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
