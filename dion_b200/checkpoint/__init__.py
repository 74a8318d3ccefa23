"""Distributed checkpointing (torch.distributed.checkpoint, DCP).

The optimizer state goes through the container's DCP-flattened
``state_dict`` (keys ``state.<fqn>.<key>`` / ``param_groups.<fqn>.<hyper>``,
as ada_dion/integration/hybrid_optimizer.py:288-307 produces), the model
through ``get_model_state_dict``, so checkpoints reshard across world sizes
like torchtitan's CheckpointManager (interval, optional model-only final
save). Before every save, Dion-family optimizers with a replicate mesh
average their state across replicas (``synchronize_for_checkpoint``), which
the reference container never calls.
"""
from __future__ import annotations

import os
import re
from typing import Any, Dict, Optional

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp
from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict, set_model_state_dict

__all__ = ["CheckpointManager", "save", "load"]


def _sync_for_checkpoint(optimizers) -> None:
    for opt in getattr(optimizers, "optimizers", [optimizers]):
        fn = getattr(opt, "synchronize_for_checkpoint", None)
        if fn is not None:
            fn()


def save(folder: str, model, optimizers, step: int, model_only: bool = False, data=None) -> str:
    """Write a DCP checkpoint. Full checkpoints go to ``step-<N>``; a
    model-only save goes to ``step-<N>-model``, a name that resuming never
    picks (it holds no optimizer state to resume from). ``data``: a loader
    with ``state_dict()`` (the global samples consumed), stored beside the
    step so a resumed job continues at the same sample."""
    path = os.path.join(folder, f"step-{step}-model" if model_only else f"step-{step}")
    _sync_for_checkpoint(optimizers)
    sd: Dict[str, Any] = {"model": get_model_state_dict(model)}
    if not model_only:
        sd["optimizer"] = optimizers.state_dict()
        sd["train_state"] = {"step": torch.tensor(step)}
        if data is not None and hasattr(data, "state_dict"):
            sd["train_state"]["data_samples"] = torch.tensor(int(data.state_dict()["samples"]))
    dcp.save(sd, checkpoint_id=path)
    return path


def _metadata_keys(path: str):
    return dcp.FileSystemReader(path).read_metadata().state_dict_metadata.keys()


def _has_optimizer_state(path: str) -> bool:
    """Whether the checkpoint at ``path`` holds optimizer entries (a
    model-only save does not); read from the DCP metadata only."""
    return any(k.startswith("optimizer.") for k in _metadata_keys(path))


def load(path: str, model, optimizers=None, data=None) -> int:
    """Load model (and, when the checkpoint has them, optimizer, step and
    data position) state; returns the saved step, 0 for a model-only
    checkpoint. Errors in loading the optimizer state are raised, never
    skipped. ``data``: a loader with ``load_state_dict``; checkpoints written
    without a data position leave it where it is."""
    sd: Dict[str, Any] = {"model": get_model_state_dict(model)}
    keys = set(_metadata_keys(path))
    has_opt = optimizers is not None and any(k.startswith("optimizer.") for k in keys)
    has_data = has_opt and data is not None and "train_state.data_samples" in keys
    if has_opt:
        sd["optimizer"] = optimizers.state_dict()
        sd["train_state"] = {"step": torch.tensor(0)}
        if has_data:
            sd["train_state"]["data_samples"] = torch.tensor(0)
    dcp.load(sd, checkpoint_id=path)
    set_model_state_dict(model, sd["model"])
    if has_opt:
        optimizers.load_state_dict(sd["optimizer"])
        if has_data:
            data.load_state_dict({"samples": int(sd["train_state"]["data_samples"])})
        return int(sd["train_state"]["step"])
    return 0


class CheckpointManager:
    def __init__(self, folder: str, model, optimizers, interval: int = 1000, model_only_last: bool = True):
        self.folder = folder
        self.model = model
        self.optimizers = optimizers
        self.interval = interval
        self.model_only_last = model_only_last

    def latest(self) -> Optional[str]:
        """Newest full checkpoint (``step-<N>``); model-only final saves
        (``step-<N>-model``) are not resume points."""
        if not os.path.isdir(self.folder):
            return None
        steps = [int(m.group(1)) for d in os.listdir(self.folder) if (m := re.fullmatch(r"step-(\d+)", d))]
        return os.path.join(self.folder, f"step-{max(steps)}") if steps else None

    def maybe_load(self, trainer) -> None:
        p = self.latest()
        if p is not None:
            trainer.step_idx = load(p, self.model, self.optimizers, data=getattr(trainer, "data", None))

    def maybe_save(self, trainer, step: int, final: bool = False) -> Optional[str]:
        """Full checkpoint every ``interval`` steps (the final step included);
        the final step additionally gets a model-only export when
        ``model_only_last``, or a full checkpoint when that step is off the
        interval and ``model_only_last`` is False."""
        path = None
        data = getattr(trainer, "data", None)
        if self.interval > 0 and step % self.interval == 0:
            path = save(self.folder, self.model, self.optimizers, step, data=data)
        if final:
            if self.model_only_last:
                path = save(self.folder, self.model, self.optimizers, step, model_only=True)
            elif path is None:
                path = save(self.folder, self.model, self.optimizers, step, data=data)
        return path
