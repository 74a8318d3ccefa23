"""Dion (or any dion_b200 optimizer) in a plain PyTorch training loop.

    python examples/plain_pytorch.py --optimizer dion --steps 200 [--device cuda]

Matrices go to the orthonormalising optimizer; embeddings, norms and the
output head to its built-in AdamW (an ``algorithm: adamw`` parameter group),
the grouping the reference's container uses. The model is a small Llama from
this package; any ``nn.Module`` works the same way.
"""
import argparse

import torch

from dion_b200.integration.param_grouper import group_params_for_hybrid
from dion_b200.models.llama3 import Transformer, llama3_config
from dion_b200.optim import AdaDionV2, Dion, Dion2, Muon


def make_optimizer(name: str, model: torch.nn.Module, lr: float):
    g = group_params_for_hybrid(model)
    scalar = dict(algorithm="adamw", lr=3e-4, betas=(0.9, 0.95), weight_decay=0.01)
    groups = [{"params": g.matrix_params},
              {"params": g.embed_params + g.norm_params, **scalar},
              {"params": g.output_params, **scalar, "lr": 3e-4 / model.cfg.dim ** 0.5}]
    if name == "muon":
        return Muon(groups, lr=lr)
    if name == "dion":
        return Dion(groups, lr=lr, rank_fraction=0.25)
    if name == "dion2":
        return Dion2(groups, lr=lr, fraction=0.25)
    if name == "adadion_v2":
        return AdaDionV2(groups, lr=lr, adaptive_rank=True, rank_fraction_max=0.5, init_rank_fraction=0.25)
    raise SystemExit(f"unknown optimizer {name}")


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--optimizer", default="dion", choices=["muon", "dion", "dion2", "adadion_v2"])
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--lr", type=float, default=0.02)
    p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = p.parse_args(argv)
    torch.manual_seed(0)
    dev = torch.device(a.device)
    cfg = llama3_config("tiny", vocab_size=512, max_seq_len=64)
    with dev:
        model = Transformer(cfg)
    model.init_weights()
    if dev.type == "cuda":
        model = model.to(torch.bfloat16)
    opt = make_optimizer(a.optimizer, model, a.lr)
    # a fixed batch to memorise: the loss must fall
    data = torch.randint(0, cfg.vocab_size, (8, 65), generator=torch.Generator().manual_seed(1)).to(dev)
    losses = []
    for step in range(a.steps):
        loss = model.loss(data[:, :-1], data[:, 1:])
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(float(loss.detach()))
        if step % 20 == 0 or step == a.steps - 1:
            print(f"step {step:4d}  loss {losses[-1]:.4f}", flush=True)
    return losses


if __name__ == "__main__":
    main()
