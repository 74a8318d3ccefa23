"""FSDP2 / HSDP application for the Llama model.

Mirrors what torchtitan's parallelize_llama does for data parallelism
(referenced by ada_dion/integration/config_registry.py:92-103): one
``fully_shard`` unit per transformer block plus a root unit holding the
embedding, final norm and LM head; bf16 parameters for compute and fp32 for
the gradient reduce-scatter. With a 2-D (replicate, shard) mesh this is
HSDP.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
from torch.distributed.device_mesh import DeviceMesh
from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard

__all__ = ["apply_fsdp"]


def apply_fsdp(
    model: nn.Module,
    mesh: DeviceMesh,
    param_dtype: torch.dtype = torch.bfloat16,
    reduce_dtype: torch.dtype = torch.float32,
    reshard_after_forward: bool = True,
) -> nn.Module:
    # activations are already bf16 (the embedding runs in param_dtype); keeping
    # forward inputs uncast leaves the fp32 rotary table intact
    mp = MixedPrecisionPolicy(param_dtype=param_dtype, reduce_dtype=reduce_dtype, cast_forward_inputs=False)
    layers = list(model.layers.values()) if isinstance(model.layers, nn.ModuleDict) else list(model.layers)
    for i, block in enumerate(layers):
        # the last block is resharded by the root right after backward anyway
        fully_shard(block, mesh=mesh, mp_policy=mp, shard_placement_fn=_fsdp_placement,
                    reshard_after_forward=reshard_after_forward and i < len(layers) - 1)
    fully_shard(model, mesh=mesh, mp_policy=mp, reshard_after_forward=reshard_after_forward,
                shard_placement_fn=_fsdp_placement)
    return model


def _fsdp_placement(param: nn.Parameter):
    """FSDP shards dim 0, except for weights tensor parallelism already splits
    along dim 0 (column-parallel): those are sharded along dim 1 so each
    matrix has one mesh per dimension (no strided sharding), which is the
    layout Dion's FSDP x TP update expects (ada_dion/optim/adadion_v2.py:572-575
    rejects the strided form)."""
    from torch.distributed.tensor import DTensor, Shard

    if isinstance(param, DTensor) and param.ndim == 2:
        if any(pl.is_shard() and pl.dim == 0 for pl in param.placements):
            return Shard(1)
    return Shard(0)
