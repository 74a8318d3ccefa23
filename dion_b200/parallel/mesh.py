"""Device-mesh construction for (replicate, shard, tp) layouts.

The optimizer receives the real sub-meshes: the FSDP shard sub-mesh as
``outer_shard_mesh`` / ``distributed_mesh``, the replicate sub-mesh for HSDP
and the TP sub-mesh as ``inner_shard_mesh``. (The reference container passes
a 1-D world mesh in every case, ada_dion/integration/hybrid_optimizer.py:
39-48, which its Dion rejects under HSDP.)
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh, init_device_mesh

__all__ = ["ParallelDims", "init_distributed", "build_mesh"]


@dataclass
class ParallelDims:
    dp_replicate: int = 1
    dp_shard: int = -1
    tp: int = 1
    pp: int = 1

    def resolve(self, world: int) -> "ParallelDims":
        shard = self.dp_shard
        if shard == -1:
            shard = world // (self.dp_replicate * self.tp * self.pp)
        if self.dp_replicate * shard * self.tp * self.pp != world:
            raise ValueError(
                f"parallel dims {self.dp_replicate}x{shard}x{self.tp}x{self.pp} != world size {world}"
            )
        return ParallelDims(self.dp_replicate, shard, self.tp, self.pp)


def init_distributed(backend: Optional[str] = None, timeout_s: float = 300.0) -> tuple[int, int, int]:
    """Initialise torch.distributed from torchrun's environment (single process if absent)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    if not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        import datetime

        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        if world == 1 and "MASTER_ADDR" not in os.environ:
            # single process: a private in-memory store, no rendezvous
            kw["store"] = dist.HashStore()
            kw["rank"] = 0
            kw["world_size"] = 1
        restart = int(os.environ.get("TORCHELASTIC_RESTART_COUNT", "0") or 0)
        if world > 1 and restart > 0 and "MASTER_ADDR" in os.environ:
            # an elastic restart: the launcher's store still holds the failed attempt's
            # process-group keys (peer addresses, communicator ids), which a rank could
            # read before its new peer overwrites them; key this attempt apart
            agent_store = os.environ.get("TORCHELASTIC_USE_AGENT_STORE") == "True"
            base = dist.TCPStore(os.environ["MASTER_ADDR"], int(os.environ["MASTER_PORT"]), world,
                                 is_master=not agent_store and rank == 0,
                                 timeout=datetime.timedelta(seconds=timeout_s))
            kw.update(store=dist.PrefixStore(f"dion_b200/attempt_{restart}", base), rank=rank, world_size=world)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world, local


def build_mesh(dims: ParallelDims, device_type: Optional[str] = None) -> Optional[DeviceMesh]:
    """Mesh with named dims ("dp_replicate", "dp_shard", "tp", "pp"), size-1 dims
    dropped -- except ``dp_shard`` beside a replicate or TP dim: replicas
    without sharding are HSDP with a shard dim of 1 (FSDP2 then all-reduces
    the gradients over the replicas and every replica holds whole matrices),
    and TP without data parallelism still gets FSDP2's mixed precision."""
    world = dist.get_world_size() if dist.is_initialized() else 1
    d = dims.resolve(world)
    if device_type is None:
        device_type = "cuda" if torch.cuda.is_available() else "cpu"
    names, sizes = [], []
    for name, size in (("pp", d.pp), ("dp_replicate", d.dp_replicate), ("dp_shard", d.dp_shard), ("tp", d.tp)):
        # dp_shard stays (size 1) beside a replicate or TP dim: FSDP2 then still
        # applies (mixed precision: bf16 compute, fp32 master weights) when every
        # rank of a TP group holds the whole data-parallel shard
        if size > 1 or (name == "dp_shard" and (d.dp_replicate > 1 or d.tp > 1)):
            names.append(name)
            sizes.append(size)
    if not names:
        names, sizes = ["dp_shard"], [1]
    return init_device_mesh(device_type, tuple(sizes), mesh_dim_names=tuple(names))
