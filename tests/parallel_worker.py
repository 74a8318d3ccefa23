"""Worker for tests/test_parallel_gpu.py: run under torchrun, one rank per GPU.

Trains a small Llama with the package's trainer on a given layout
(dp_replicate x dp_shard x tp) over NCCL and prints, from rank 0, one JSON
line with the per-step losses and the largest device status word seen.

    python -m torch.distributed.run --nproc-per-node 2 tests/parallel_worker.py Muon 2 1 1
"""
import json
import sys

import torch
import torch.distributed as dist


def main():
    optimizer, rep, shard, tp = sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4])
    local_batch = int(sys.argv[5]) if len(sys.argv) > 5 else 2
    from dion_b200 import ops
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig
    from dion_b200.parallel.mesh import init_distributed

    init_distributed(timeout_s=120.0)
    opt = HybridOptimizersContainer.Config(name=optimizer, lr=0.02, scalar_lr=3e-3)
    cfg = TrainerConfig(model="tiny", model_overrides=dict(n_layers=2, vocab_size=512, max_seq_len=128),
                        seq_len=64, local_batch_size=local_batch, steps=4, warmup_steps=0, dp_replicate=rep,
                        dp_shard=shard, tp=tp, optimizer=opt, seed=5)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=None if torch.cuda.is_available() else torch.device("cpu"))
    losses = []
    for _ in range(4):
        t, l = tr.data.next()
        losses.append(float(tr.train_step(t, l)))
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    status = ops.ext().status_read() if torch.cuda.is_available() and ops.has_ext() else 0
    if dist.get_rank() == 0:
        print(json.dumps({"optimizer": optimizer, "layout": [rep, shard, tp], "world": dist.get_world_size(),
                          "losses": losses, "status": status}), flush=True)
    from dion_b200.parallel.symm import release_all

    release_all()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
