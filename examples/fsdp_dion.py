"""Dion under FSDP2 in your own training loop (one process per GPU).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/fsdp_dion.py --steps 100
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/fsdp_dion.py --steps 3   # CPU: gloo

The model is sharded with FSDP2 over a 1-D mesh; Dion gets the same mesh as
``outer_shard_mesh`` and works on the sharded matrices directly (its P
reduce-scatter / all-gather run inside its GEMMs over NVLink on one node).
Embeddings, norms and the output head use Dion's built-in AdamW.
"""
import argparse
import os

import torch
import torch.distributed as dist
from torch.distributed.device_mesh import init_device_mesh

from dion_b200.integration.param_grouper import group_params_for_hybrid
from dion_b200.models.llama3 import Transformer, llama3_config
from dion_b200.optim import Dion
from dion_b200.parallel.fsdp import apply_fsdp


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--lr", type=float, default=0.02)
    a = p.parse_args(argv)
    cuda = torch.cuda.is_available()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if cuda:
        torch.cuda.set_device(local)
    dist.init_process_group("nccl" if cuda else "gloo")
    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", local) if cuda else torch.device("cpu")
    mesh = init_device_mesh(dev.type, (world,), mesh_dim_names=("dp_shard",))

    torch.manual_seed(0)
    cfg = llama3_config("tiny", vocab_size=512, max_seq_len=64)
    with dev:
        model = Transformer(cfg)
    model.init_weights()
    apply_fsdp(model, mesh)  # bf16 compute, fp32 master weights and gradient reduction

    g = group_params_for_hybrid(model)
    scalar = dict(algorithm="adamw", lr=3e-4, betas=(0.9, 0.95), weight_decay=0.01)
    opt = Dion([{"params": g.matrix_params},
                {"params": g.embed_params + g.norm_params + g.output_params, **scalar}],
               outer_shard_mesh=mesh, lr=a.lr, rank_fraction=0.25)

    gen = torch.Generator().manual_seed(1 + rank)  # each rank its own sequences
    data = torch.randint(0, cfg.vocab_size, (4, 65), generator=gen).to(dev)
    for step in range(a.steps):
        loss = model.loss(data[:, :-1], data[:, 1:])
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        avg = loss.detach().clone()
        dist.all_reduce(avg)
        if rank == 0 and (step % 10 == 0 or step == a.steps - 1):
            print(f"step {step:4d}  loss {float(avg) / world:.4f}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
