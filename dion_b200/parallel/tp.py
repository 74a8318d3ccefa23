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

__all__ = ["apply_tp", "sp_sync_replicated_grads", "TP_PLAN"]

TP_PLAN = {
    "attention.wq": "colwise",
    "attention.wk": "colwise",
    "attention.wv": "colwise",
    "attention.wo": "rowwise",
    "feed_forward.w1": "colwise",
    "feed_forward.w3": "colwise",
    "feed_forward.w2": "rowwise",
}


def apply_tp(model: nn.Module, tp_mesh: DeviceMesh, sequence_parallel: bool = False) -> nn.Module:
    """Shard the block weights over ``tp_mesh`` (the plan above). With
    ``sequence_parallel`` the activations between sublayers are token shards
    and the TP collectives run fused into the GEMMs (parallel/sp.py); the
    weights are distributed identically either way, so optimizer state and
    checkpoints do not depend on the choice."""
    tp = tp_mesh.size()
    cfg = getattr(model, "cfg", None)
    if cfg is not None and (cfg.n_heads % tp or cfg.kv_heads % tp):
        raise ValueError(f"heads ({cfg.n_heads}/{cfg.kv_heads}) must be divisible by the TP degree {tp}")
    layers = model.layers.values() if isinstance(model.layers, nn.ModuleDict) else model.layers
    for block in layers:
        plan = {k: (ColwiseParallel() if v == "colwise" else RowwiseParallel()) for k, v in TP_PLAN.items()}
        parallelize_module(block, tp_mesh, plan)
    if sequence_parallel:
        import torch

        from .sp import SPGroup

        dev = next(model.parameters()).device
        sp = SPGroup(tp_mesh.get_group(), dev if dev.type != "meta" else torch.device("cuda"))
        model.sp = sp
        for block in layers:
            block.attention.sp = sp
            block.feed_forward.sp = sp
    return model


def sp_sync_replicated_grads(model: nn.Module, group) -> None:
    """Sum, over the TP group, the gradients of parameters that TP does not
    shard (embedding, norms, LM head): under sequence parallelism each TP rank
    back-propagates only its own tokens through them. One coalesced
    all-reduce."""
    import torch
    import torch.distributed as dist
    from torch.distributed.tensor import DTensor

    grads = []
    for p in model.parameters():
        if p.grad is None:
            continue
        if isinstance(p, DTensor) and "tp" in (p.device_mesh.mesh_dim_names or ()):
            continue
        g = p.grad
        grads.append(g.to_local() if isinstance(g, DTensor) else g)
    if not grads:
        return
    by_dtype = {}
    for g in grads:
        by_dtype.setdefault(g.dtype, []).append(g)
    for gs in by_dtype.values():
        flat = torch.cat([g.reshape(-1) for g in gs])
        dist.all_reduce(flat, group=group)
        off = 0
        for g in gs:
            g.copy_(flat[off:off + g.numel()].view_as(g))
            off += g.numel()
