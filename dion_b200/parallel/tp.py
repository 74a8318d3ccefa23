"""Tensor parallelism for the Llama model (Megatron-style column/row split).

Per transformer block: wq, wk, wv, w1, w3 are column-parallel (output
features sharded, ``Shard(0)`` of the weight on the TP mesh) and wo, w2 are
row-parallel (input features sharded, ``Shard(1)``), so each block needs one
all-reduce after attention and one after the MLP in the forward (and their
mirrors in the backward). Embedding, norms and the LM head stay replicated
over TP. This is the plan torchtitan's parallelize_llama applies when
``--parallelism.tensor_parallel_degree`` > 1, which the reference's configs
register but never enable (ada_dion/integration/config_registry.py:92-103).

Apply before FSDP so FSDP shards the TP-local tensors over the data-parallel
mesh (2-D FSDP x TP parameters). Local head counts must divide evenly:
``n_heads % tp == 0`` and ``n_kv_heads % tp == 0``.
"""
from __future__ import annotations

import torch.nn as nn
from torch.distributed.device_mesh import DeviceMesh
from torch.distributed.tensor.parallel import ColwiseParallel, RowwiseParallel, parallelize_module

__all__ = ["apply_tp", "TP_PLAN"]

TP_PLAN = {
    "attention.wq": "colwise",
    "attention.wk": "colwise",
    "attention.wv": "colwise",
    "attention.wo": "rowwise",
    "feed_forward.w1": "colwise",
    "feed_forward.w3": "colwise",
    "feed_forward.w2": "rowwise",
}


def apply_tp(model: nn.Module, tp_mesh: DeviceMesh) -> nn.Module:
    tp = tp_mesh.size()
    cfg = getattr(model, "cfg", None)
    if cfg is not None and (cfg.n_heads % tp or cfg.kv_heads % tp):
        raise ValueError(f"heads ({cfg.n_heads}/{cfg.kv_heads}) must be divisible by the TP degree {tp}")
    layers = model.layers.values() if isinstance(model.layers, nn.ModuleDict) else model.layers
    for block in layers:
        plan = {k: (ColwiseParallel() if v == "colwise" else RowwiseParallel()) for k, v in TP_PLAN.items()}
        parallelize_module(block, tp_mesh, plan)
    return model
