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
from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp
from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict, set_model_state_dict
from torch.distributed.tensor import DTensor, distribute_tensor

__all__ = ["CheckpointManager", "save", "load"]


def _sync_for_checkpoint(optimizers) -> None:
    for opt in getattr(optimizers, "optimizers", [optimizers]):
        fn = getattr(opt, "synchronize_for_checkpoint", None)
        if fn is not None:
            fn()


def save(folder: str, model, optimizers, step: int, model_only: bool = False, data=None,
         async_save: bool = False, process_group=None, export_dtype: Optional[torch.dtype] = None):
    """Write a DCP checkpoint. Full checkpoints go to ``step-<N>``; a
    model-only save goes to ``step-<N>-model``, a name that resuming never
    picks (it holds no optimizer state to resume from). ``data``: a loader
    with ``state_dict()`` (the global samples consumed), stored beside the
    step so a resumed job continues at the same sample."""
    path = os.path.join(folder, f"step-{step}-model" if model_only else f"step-{step}")
    _sync_for_checkpoint(optimizers)
    sd: Dict[str, Any] = {"model": get_model_state_dict(model)}
    if model_only and export_dtype is not None:  # e.g. bf16 weights for an export
        sd["model"] = {k: v.to(export_dtype) if torch.is_tensor(v) and v.is_floating_point() else v
                       for k, v in sd["model"].items()}
    if not model_only:
        sd["optimizer"] = optimizers.state_dict()
        sd["train_state"] = {"step": torch.tensor(step)}
        if data is not None and hasattr(data, "state_dict"):
            sd["train_state"]["data_samples"] = torch.tensor(int(data.state_dict()["samples"]))
    if async_save:
        # the state is staged to host memory before this returns; the files are
        # written in the background while training continues (a future). Each
        # tensor is copied into its own storage first: optimizer state lives in
        # views of shared arenas, which the stager cannot copy storage-wise.
        return path, dcp.async_save(_own_storage(sd), checkpoint_id=path, process_group=process_group)
    dcp.save(sd, checkpoint_id=path)
    return path


def _own_storage(obj):
    if isinstance(obj, dict):
        return {k: _own_storage(v) for k, v in obj.items()}
    if isinstance(obj, list):
        return [_own_storage(v) for v in obj]
    if torch.is_tensor(obj):
        return obj.detach().clone()
    return obj


def _metadata_keys(path: str):
    return dcp.FileSystemReader(path).read_metadata().state_dict_metadata.keys()


def _has_optimizer_state(path: str) -> bool:
    """Whether the checkpoint at ``path`` holds optimizer entries (a
    model-only save does not); read from the DCP metadata only."""
    return any(k.startswith("optimizer.") for k in _metadata_keys(path))


def _reoriented_q_entries(opt_sd: Dict[str, Any], path: str) -> List[Tuple[str, Any]]:
    """Dion-family ``Q`` entries saved on the other side of their matrix.

    Dion keeps Q (rows x rank) on the side of the matrix its sharding
    dictates, so a layout change (for example FSDP x TP -> one process) can
    flip it: saved [n, r] where this layout wants [m, r], or the reverse.
    Those entries are loaded whole (a plain tensor of the saved shape) and
    converted by :func:`_convert_reoriented_q`; returns (key, this layout's
    template) pairs."""
    md = dcp.FileSystemReader(path).read_metadata().state_dict_metadata
    todo = []
    for k, t in list(opt_sd.items()):
        if not (k.startswith("state.") and k.endswith(".Q") and torch.is_tensor(t) and t.dim() == 2):
            continue
        meta = md.get("optimizer." + k)
        saved = tuple(getattr(meta, "size", ()) or ())
        if len(saved) != 2 or saved == tuple(t.shape) or saved[1] != t.shape[1]:
            continue
        local = t.to_local() if isinstance(t, DTensor) else t
        opt_sd[k] = torch.empty(saved, dtype=t.dtype, device=local.device)
        todo.append((k, t))
    return todo


def _convert_reoriented_q(opt_sd: Dict[str, Any], todo: List[Tuple[str, Any]]) -> None:
    """Q on the other side of M: the column-normalised M Q (or M^T Q), the
    estimate of that side's subspace the power iteration would form next
    (Dion: P = M Q, then R = M^T orth(P) -> Q). Every rank computes it from
    the whole M and keeps its own shard."""
    for k, template in todo:
        M = opt_sd[k[: -len("Q")] + "momentum"]
        M = (M.full_tensor() if isinstance(M, DTensor) else M).float()
        Qs = opt_sd[k].float().to(M.device)
        P = M @ Qs if Qs.shape[0] == M.shape[1] else M.t() @ Qs
        Q = (P / P.norm(dim=0, keepdim=True).clamp_min(1e-12)).to(template.dtype)
        if tuple(Q.shape) != tuple(template.shape):
            raise ValueError(f"{k}: saved Q {tuple(Qs.shape)} fits neither side of its momentum {tuple(M.shape)}")
        if isinstance(template, DTensor):
            Q = distribute_tensor(Q, template.device_mesh, template.placements, src_data_rank=None)
        opt_sd[k] = Q


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
    reoriented: List[Tuple[str, Any]] = []
    if has_opt:
        sd["optimizer"] = optimizers.state_dict()
        reoriented = _reoriented_q_entries(sd["optimizer"], path)
        sd["train_state"] = {"step": torch.tensor(0)}
        if has_data:
            sd["train_state"]["data_samples"] = torch.tensor(0)
    dcp.load(sd, checkpoint_id=path)
    set_model_state_dict(model, sd["model"])
    if has_opt:
        _convert_reoriented_q(sd["optimizer"], reoriented)
        optimizers.load_state_dict(sd["optimizer"])
        if has_data:
            data.load_state_dict({"samples": int(sd["train_state"]["data_samples"])})
        return int(sd["train_state"]["step"])
    return 0


class CheckpointManager:
    """Interval checkpoints of a trainer. ``async_mode`` "async": each save
    returns once the state is staged in host memory and the files are written
    in the background (torchtitan's async checkpointing); the next save, and
    :meth:`wait`, wait for the previous write."""

    def __init__(self, folder: str, model, optimizers, interval: int = 1000, model_only_last: bool = True,
                 async_mode: str = "disabled", export_dtype: Optional[torch.dtype] = None):
        if async_mode not in ("disabled", "async"):
            raise ValueError(f"async_mode must be 'disabled' or 'async', got {async_mode!r}")
        self.folder = folder
        self.model = model
        self.optimizers = optimizers
        self.interval = interval
        self.model_only_last = model_only_last
        self.async_mode = async_mode
        self.export_dtype = export_dtype  # dtype of the model-only final export (None: as trained)
        self._pending = None
        self._pg = None
        if async_mode == "async" and dist.is_initialized() and dist.get_world_size() > 1:
            # the background write coordinates the ranks on a group of its own, so
            # it never interleaves with the training step's collectives
            self._pg = dist.new_group(backend="gloo")

    def wait(self) -> None:
        """Block until the last background write has finished."""
        if self._pending is not None:
            self._pending.result()
            self._pending = None

    def _save(self, step: int, model_only: bool = False, data=None) -> str:
        self.wait()
        dt = self.export_dtype if model_only else None
        if self.async_mode == "async":
            path, self._pending = save(self.folder, self.model, self.optimizers, step, model_only=model_only,
                                       data=data, async_save=True, process_group=self._pg, export_dtype=dt)
            return path
        return save(self.folder, self.model, self.optimizers, step, model_only=model_only, data=data,
                    export_dtype=dt)

    def latest(self) -> Optional[str]:
        """Newest full checkpoint (``step-<N>``); model-only final saves
        (``step-<N>-model``) are not resume points."""
        if not os.path.isdir(self.folder):
            return None
        steps = [int(m.group(1)) for d in os.listdir(self.folder) if (m := re.fullmatch(r"step-(\d+)", d))]
        return os.path.join(self.folder, f"step-{max(steps)}") if steps else None

    def maybe_load(self, trainer, load_step: int = -1, initial_load_path: Optional[str] = None,
                   initial_load_model_only: bool = True) -> Optional[str]:
        """Resume from ``step-<load_step>`` (or, with -1, the newest full
        checkpoint in the folder); with no checkpoint in the folder, start
        from ``initial_load_path`` (its weights only, unless
        ``initial_load_model_only`` is False). Returns the path loaded."""
        self.wait()
        if load_step >= 0:
            p = os.path.join(self.folder, f"step-{load_step}")
            if not os.path.isdir(p):
                raise FileNotFoundError(f"no checkpoint {p}")
        else:
            p = self.latest()
        data = getattr(trainer, "data", None)
        if p is not None:
            trainer.step_idx = load(p, self.model, self.optimizers, data=data)
            return p
        if initial_load_path:
            if initial_load_model_only:
                load(initial_load_path, self.model, None)
            else:
                trainer.step_idx = load(initial_load_path, self.model, self.optimizers, data=data)
            return initial_load_path
        return None

    def maybe_save(self, trainer, step: int, final: bool = False) -> Optional[str]:
        """Full checkpoint every ``interval`` steps (the final step included);
        the final step additionally gets a model-only export when
        ``model_only_last``, or a full checkpoint when that step is off the
        interval and ``model_only_last`` is False."""
        path = None
        data = getattr(trainer, "data", None)
        if self.interval > 0 and step % self.interval == 0:
            path = self._save(step, data=data)
        if final:
            if self.model_only_last:
                path = self._save(step, model_only=True)
            elif path is None:
                path = self._save(step, data=data)
            self.wait()
        return path
