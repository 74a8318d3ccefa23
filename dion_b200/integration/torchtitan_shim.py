"""Run this package's optimizers inside torchtitan's own trainer.

Importing this module registers a train spec ``dion_b200_llama3``: torchtitan's
Llama-3 model, parallelisation, data and loss, with the optimizer builder
replaced by :func:`build_dion_optimizers` (this package's
:class:`HybridOptimizersContainer`: Muon / Dion / Dion2 / AdaDion /
AdaDionV2 on the matrices, AdamW on embeddings, norms and the output head).
It also extends torchtitan's ``[optimizer]`` section with the Dion-family
hyper-parameters. The reference reaches torchtitan the same way through its
experiment shim (torchtitan_shim/config_registry.py, scripts/patch_torchtitan.sh);
here nothing in torchtitan is patched:

    python -m torchtitan.train \\
        --experimental.custom_import dion_b200.integration.torchtitan_shim \\
        --experimental.custom_args_module dion_b200.integration.torchtitan_shim \\
        --model.name dion_b200_llama3 --model.flavor debugmodel \\
        --optimizer.name Dion --optimizer.lr 0.02 --optimizer.rank_fraction 0.25
"""
# (no ``from __future__ import annotations``: torchtitan's config merge
# inspects the dataclass field types, which must be classes, not strings)
import dataclasses
from dataclasses import dataclass, field
from typing import Any, List, Optional

import torch.nn as nn

from .hybrid_optimizer import HybridOptimizersContainer

__all__ = ["Optimizer", "JobConfig", "build_dion_optimizers", "register", "TRAIN_SPEC_NAME"]

TRAIN_SPEC_NAME = "dion_b200_llama3"
_NAMES = {"muon": "Muon", "dion": "Dion", "dion2": "Dion2", "adadion": "AdaDion", "adadion_v2": "AdaDionV2",
          "adadionv2": "AdaDionV2", "adamw": "AdamW"}


_SCALARS = {"float": float, "int": int, "bool": bool, "str": str, float: float, int: int, bool: bool, str: str}
# torchtitan's own [optimizer] fields, read separately
_TITAN_OWNED = {"name", "lr", "weight_decay", "scalar_beta1", "scalar_beta2", "scalar_eps"}

# Fields merged into torchtitan's ``[optimizer]`` section: every scalar field of
# the container's Config (Dion / Dion2 / AdaDion / AdaDionV2 / GSDion switches),
# so each one is settable from torchtitan's command line.
def _field_class(f):
    if f.type in _SCALARS:
        return _SCALARS[f.type]
    if f.type in ("Optional[str]", Optional[str]) and isinstance(f.default, str):
        return str  # e.g. adjust_lr: a name, or None to switch it off
    return None


Optimizer = dataclasses.make_dataclass(
    "Optimizer",
    [(f.name, _field_class(f), field(default=f.default))
     for f in dataclasses.fields(HybridOptimizersContainer.Config)
     if f.name not in _TITAN_OWNED and _field_class(f) is not None and f.default is not dataclasses.MISSING],
)
Optimizer.__doc__ = "Fields merged into torchtitan's ``[optimizer]`` section."


@dataclass
class JobConfig:
    optimizer: Optimizer = field(default_factory=Optimizer)


def _container_config(oc: Any) -> HybridOptimizersContainer.Config:
    name = _NAMES.get(str(oc.name).lower().replace("-", "_"))
    if name is None:
        raise ValueError(f"{oc.name!r} is not a dion_b200 optimizer ({sorted(set(_NAMES.values()))})")
    cfg = HybridOptimizersContainer.Config(name=name, lr=float(oc.lr), weight_decay=float(oc.weight_decay))
    for f in dataclasses.fields(Optimizer):
        if hasattr(oc, f.name) and hasattr(cfg, f.name):
            setattr(cfg, f.name, getattr(oc, f.name))
    cfg.scalar_beta1, cfg.scalar_beta2 = float(oc.beta1), float(oc.beta2)
    cfg.scalar_eps = float(oc.eps)
    return cfg


def build_dion_optimizers(model_parts: List[nn.Module], optimizer_config: Any, parallel_dims: Any,
                          ft_manager: Optional[Any] = None) -> HybridOptimizersContainer:
    """torchtitan ``build_optimizers_fn``: meshes from torchtitan's world mesh
    (FSDP: ``dp_shard_cp``, HSDP replicas: ``dp_replicate``, TP: ``tp``)."""
    shard = replicate = tp = None
    if getattr(parallel_dims, "world_size", 1) > 1:
        mesh = parallel_dims.world_mesh
        names = set(mesh.mesh_dim_names or ()) | set(getattr(mesh, "_flatten_mapping", {}) or {})
        if getattr(parallel_dims, "dp_shard_enabled", False) or getattr(parallel_dims, "cp_enabled", False):
            shard = mesh["dp_shard_cp"]
        if getattr(parallel_dims, "dp_replicate_enabled", False) and "dp_replicate" in names:
            replicate = mesh["dp_replicate"]
        if getattr(parallel_dims, "tp_enabled", False):
            tp = mesh["tp"]
    return HybridOptimizersContainer(_container_config(optimizer_config), model_parts=model_parts, shard_mesh=shard,
                                     replicate_mesh=replicate, tp_mesh=tp)


def register() -> bool:
    """Register the ``dion_b200_llama3`` train spec (idempotent). False when torchtitan is absent."""
    try:
        import torchtitan.models  # noqa: F401  (registers the built-in specs)
        from torchtitan.protocols.train_spec import _train_specs, get_train_spec, register_train_spec
    except Exception:  # noqa: BLE001
        return False
    if TRAIN_SPEC_NAME in _train_specs:
        return True
    base = get_train_spec("llama3")
    register_train_spec(dataclasses.replace(base, name=TRAIN_SPEC_NAME, build_optimizers_fn=build_dion_optimizers))
    return True


register()
