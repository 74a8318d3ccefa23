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
        fully_shard(block, mesh=mesh, mp_policy=mp,
                    reshard_after_forward=reshard_after_forward and i < len(layers) - 1)
    fully_shard(model, mesh=mesh, mp_policy=mp, reshard_after_forward=reshard_after_forward)
    return model
