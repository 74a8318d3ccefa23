"""Loss parity against the reference implementation (same seed, data, init).

Runs this package's optimizer and the reference's (the ``ada_dion`` package
installed in baseline/_ref, and the ``dion`` package it depends on) side by
side and records both loss curves:

  python -m dion_b200.benchmarks.parity --preset tiny --optimizer dion --steps 50 \\
      --device cpu --data fixed --out parity_tiny_dion.json

Both arms start from identical weights: the reference arm's torchtitan
Llama-3 model is loaded with the state dict of this package's model after
its seeded initialisation (the parameter names are the same). Both see the
same token batches, the same parameter groups (matrices on Dion / Muon;
embeddings, norms and the LM head on AdamW), the same learning-rate
schedule (linear warm-up, then cosine to 10 %) and gradient clipping at 1.0.
What differs is the optimizer implementation, and with it the random
streams it draws (Dion's initial Q and sketch matrices), so the curves agree
statistically rather than bit for bit; ``--ref-seeds`` reruns the reference
arm with other optimizer seeds to measure that seed-to-seed spread.

Data (``--data``):
  * ``fixed``  : one batch of tokens drawn uniformly from the vocabulary
    (seed), revisited every step: the loss measures memorisation;
  * ``stream`` : a fresh uniform batch every step (loss floor ln(vocab));
  * ``markov`` : tokens from a fixed random successor map (next = perm[cur]
    with probability 0.9, else uniform), so the loss can fall well below
    ln(vocab) and the curve shows learning.

The reference arm corresponds to ada_dion/benchmarks/tier_a_correctness.py
(same-seed runs) and ada_dion/optim/adadion_v2.py:252-289 / dion/muon.py
(the optimizer steps being compared).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time
from typing import Callable, Dict, List, Tuple

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF_PATH = os.path.join(REPO, "baseline", "_ref")

__all__ = ["make_data", "run_arm", "main"]


# ---------------------------------------------------------------- data
def make_data(kind: str, steps: int, batch: int, seq: int, vocab: int, seed: int) -> Callable[[int], Tuple]:
    """Returns ``get(step) -> (tokens, labels)`` on the CPU (int64)."""
    g = torch.Generator().manual_seed(seed)
    if kind == "fixed":
        full = torch.randint(0, vocab, (batch, seq + 1), generator=g)
        return lambda s: (full[:, :-1], full[:, 1:])
    if kind == "stream":
        seqs = [torch.randint(0, vocab, (batch, seq + 1), generator=g) for _ in range(steps)]
        return lambda s: (seqs[s][:, :-1], seqs[s][:, 1:])
    if kind == "markov":
        perm = torch.randperm(vocab, generator=g)
        nseq = steps * batch  # every step's sequences generated together, one position at a time
        x = torch.empty(nseq, seq + 1, dtype=torch.long)
        x[:, 0] = torch.randint(0, vocab, (nseq,), generator=g)
        noise = torch.rand(nseq, seq, generator=g) >= 0.9
        rnd = torch.randint(0, vocab, (nseq, seq), generator=g)
        for t in range(seq):
            x[:, t + 1] = torch.where(noise[:, t], rnd[:, t], perm[x[:, t]])
        seqs = list(x.view(steps, batch, seq + 1).unbind(0))
        return lambda s: (seqs[s][:, :-1], seqs[s][:, 1:])
    raise ValueError(kind)


def lr_factor(step: int, steps: int, warmup: int, min_frac: float = 0.1) -> float:
    """Linear warm-up, then cosine decay to ``min_frac`` (torchtitan's
    warmup + cosine schedule as the reference configures it,
    ada_dion/integration/config_registry.py:171-176)."""
    if step < warmup:
        return (step + 1) / (warmup + 1)
    if steps <= warmup:
        return 1.0
    p = (step - warmup) / max(1, steps - warmup)
    return min_frac + (1 - min_frac) * 0.5 * (1 + math.cos(math.pi * p))


# ---------------------------------------------------------------- models
def _our_model(preset: str, seq: int, device, seed: int, init: str):
    from ..models.llama3 import Transformer, llama3_config

    cfg = llama3_config(preset, max_seq_len=max(seq, 16))
    torch.manual_seed(seed)
    model = Transformer(cfg)
    model.init_weights(mode=init)
    return model.to(device), cfg


def _reference_model(cfg, init_state: Dict[str, torch.Tensor], device):
    """torchtitan's Llama-3 (the reference's model family) loaded with the
    given initial weights."""
    from torchtitan.models.llama3.model.args import TransformerModelArgs
    from torchtitan.models.llama3.model.model import Transformer

    margs = TransformerModelArgs(dim=cfg.dim, n_layers=cfg.n_layers, n_heads=cfg.n_heads, n_kv_heads=cfg.kv_heads,
                                 vocab_size=cfg.vocab_size, multiple_of=cfg.multiple_of, norm_eps=cfg.norm_eps,
                                 rope_theta=cfg.rope_theta, max_seq_len=cfg.max_seq_len)
    hidden = cfg.hidden_dim()
    with torch.device(device):
        model = Transformer(margs)
    # torchtitan derives the FFN width from multiple_of / ffn_dim_multiplier; rebuild the MLPs at the
    # configured width when that differs (same names, same shapes as this package's model)
    for blk in model.layers.values():
        ff = blk.feed_forward
        if ff.w1.out_features != hidden:
            ff.w1 = torch.nn.Linear(cfg.dim, hidden, bias=False, device=device)
            ff.w2 = torch.nn.Linear(hidden, cfg.dim, bias=False, device=device)
            ff.w3 = torch.nn.Linear(cfg.dim, hidden, bias=False, device=device)
    missing, unexpected = model.load_state_dict({k: v.to(device) for k, v in init_state.items()}, strict=False)
    missing = [k for k in missing if "freqs_cis" not in k]
    if missing or unexpected:
        raise RuntimeError(f"reference model does not take the initial state: missing {missing}, "
                           f"unexpected {unexpected}")
    return model


# ---------------------------------------------------------------- optimizers
def _groups(named, matrix_names, lr_scalar, wd_scalar):
    mats = [p for n, p in named if n in matrix_names]
    rest = [p for n, p in named if n not in matrix_names]
    scalar = dict(algorithm="adamw", lr=lr_scalar, beta1=0.9, beta2=0.95, epsilon=1e-8, weight_decay=wd_scalar)
    return [{"params": mats}, {"params": rest, **scalar}]


def _matrix_names(model) -> List[str]:
    from ..integration.param_grouper import group_params_for_hybrid

    g = group_params_for_hybrid(model)
    ids = {id(p) for p in g.matrix_params}
    return [n for n, p in model.named_parameters() if id(p) in ids]


# the research variants: reference module and class for each
_LOWRANK = {"adadion": ("adadion", "AdaDion"), "sdion": ("sdion", "SDion"), "gsdion": ("gsdion", "GSDion"),
            "agdion": ("agdion", "AGDion"), "qcdion": ("qcdion", "QCDion")}


def _build_lowrank(impl: str, optimizer: str, model, matrix_names, a):
    """The AdaDion family: matrices on the variant, the rest on its built-in
    AdamW (``algorithm: adamw`` groups), the same hyper-parameters in both arms."""
    named = list(model.named_parameters())
    mats = [p for n, p in named if n in set(matrix_names)]
    rest = [p for n, p in named if n not in set(matrix_names)]
    groups = [{"params": mats}, {"params": rest, "algorithm": "adamw", "lr": a.scalar_lr,
                                 "weight_decay": a.scalar_wd}]
    mod, cls_name = _LOWRANK[optimizer]
    if impl == "ours":
        from .. import optim

        cls = getattr(optim, cls_name)
    else:
        if REF_PATH not in sys.path:
            sys.path.insert(0, REF_PATH)
        import importlib

        cls = getattr(importlib.import_module(f"ada_dion.optim.{mod}"), cls_name)
    return cls(groups, lr=a.lr, mu=a.mu, init_rank=a.init_rank, rank_min=a.rank_min, rank_max=a.rank_max,
               weight_decay=a.wd, adamw_betas=(0.9, 0.95), adamw_eps=1e-8)


def _build_optimizer(impl: str, optimizer: str, model, matrix_names, a, mesh=None):
    if optimizer in _LOWRANK:
        return _build_lowrank(impl, optimizer, model, matrix_names, a)
    named = list(model.named_parameters())
    groups = _groups(named, set(matrix_names), a.scalar_lr, a.scalar_wd)
    if impl == "ours":
        from ..optim import AdaDionV2, Dion, Muon

        if optimizer == "dion":
            return Dion(groups, outer_shard_mesh=mesh, lr=a.lr, mu=a.mu, rank_fraction=a.rank_fraction,
                        weight_decay=a.wd)
        if optimizer == "adadion_v2":
            return AdaDionV2(groups, outer_shard_mesh=mesh, lr=a.lr, mu=a.mu, rank_fraction_max=a.rank_fraction,
                             weight_decay=a.wd, adaptive_rank=True, init_rank_fraction=a.init_rank_fraction,
                             rank_min=a.rank_min)
        return Muon(groups, distributed_mesh=mesh, lr=a.lr, mu=a.mu, weight_decay=a.wd, nesterov=False,
                    adjust_lr="spectral_norm")
    if REF_PATH not in sys.path:
        sys.path.insert(0, REF_PATH)
    if optimizer in ("dion", "adadion_v2"):
        from ada_dion.optim.adadion_v2 import AdaDionV2

        # one rank: no outer shard mesh (the same call the benchmark's reference arm makes)
        if optimizer == "adadion_v2":
            return AdaDionV2(groups, lr=a.lr, mu=a.mu, rank_fraction_max=a.rank_fraction, weight_decay=a.wd,
                             adaptive_rank=True, init_rank_fraction=a.init_rank_fraction, rank_min=a.rank_min)
        return AdaDionV2(groups, lr=a.lr, mu=a.mu, rank_fraction_max=a.rank_fraction, weight_decay=a.wd)
    from dion import Muon as RefMuon

    return RefMuon(groups, fsdp_mesh_dim=0, world_mesh=mesh, distributed_mesh=mesh, lr=a.lr, mu=a.mu,
                   weight_decay=a.wd, nesterov=False, adjust_lr="spectral_norm")


def _prepare_inductor():
    """The reference's torch.compile'd optimizer code compiles CPU graphs; use
    the system C++ compiler, whose OpenMP runtime is present on this image."""
    import torch._inductor.config as inductor_config

    if os.path.exists("/usr/bin/g++"):
        inductor_config.cpp.cxx = ("/usr/bin/g++",)


def state_layout(opt, model) -> Dict[str, Dict[str, List[int]]]:
    """{parameter name: {state key: shape}} of the optimizer state."""
    names = {id(p): n for n, p in model.named_parameters()}
    out: Dict[str, Dict[str, List[int]]] = {}
    for p, st in opt.state.items():
        if id(p) not in names:
            continue
        out[names[id(p)]] = {k: list(v.shape) for k, v in st.items() if torch.is_tensor(v) and v.dim() > 0}
    return dict(sorted(out.items()))


# ---------------------------------------------------------------- one arm
def _one_rank_mesh():
    """A 1-rank NCCL process group and device mesh for FSDP2 on one GPU."""
    import datetime

    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    if not dist.is_initialized():
        dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1,
                                timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", 0))
    return init_device_mesh("cuda", (1,), mesh_dim_names=("dp_shard",))


def run_arm(impl: str, a, init_state=None, opt_seed: int = 0) -> Dict:
    """One training run; ``a.dtype``: fp32, bf16 (bf16 weights and state) or
    mixed (FSDP2 on one GPU: fp32 master weights and optimizer state, bf16
    compute, fp32 gradient reduction -- the benchmark's setting)."""
    device = torch.device(a.device)
    model, cfg = _our_model(a.preset, a.seq_len, "cpu", a.seed, a.init)
    matrix_names = _matrix_names(model)
    if init_state is None:
        init_state = {k: v.detach().clone() for k, v in model.state_dict().items()}
    mesh = _one_rank_mesh() if a.dtype == "mixed" else None
    if impl == "ours":
        model = model.to(device)
        if a.dtype == "bf16":
            model = model.to(torch.bfloat16)
        if mesh is not None:
            from ..parallel.fsdp import apply_fsdp

            apply_fsdp(model, mesh)

        def loss_fn(t, l):
            return model.loss(t, l)
    else:
        _prepare_inductor()
        model = _reference_model(cfg, init_state, device)
        if a.dtype == "bf16":
            model = model.to(torch.bfloat16)
        if mesh is not None:
            from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard

            mp = MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32)
            blocks = list(model.layers.values())
            for i, b in enumerate(blocks):
                fully_shard(b, mesh=mesh, mp_policy=mp, reshard_after_forward=i < len(blocks) - 1)
            fully_shard(model, mesh=mesh, mp_policy=mp)

        def loss_fn(t, l):
            return F.cross_entropy(model(t).flatten(0, 1).float(), l.flatten(0, 1))
    torch.manual_seed(opt_seed)  # the optimizer's own random draws (Q init, sketches)
    opt = _build_optimizer(impl, a.optimizer, model, matrix_names, a, mesh)
    base = [g["lr"] for g in opt.param_groups]
    get = make_data(a.data, a.steps, a.batch, a.seq_len, cfg.vocab_size, a.data_seed)
    losses, ranks = [], []
    t0 = time.time()
    for s in range(a.steps):
        f = lr_factor(s, a.steps, a.warmup)
        for g, b in zip(opt.param_groups, base):
            g["lr"] = b * f
        tok, lab = get(s)
        loss = loss_fn(tok.to(device), lab.to(device))
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(float(loss.detach().float().item()))
        rk = opt.get_rank() if hasattr(opt, "get_rank") else {}
        if rk:  # adaptive rank: the mean active rank over the matrices after this step
            ranks.append(sum(rk.values()) / len(rk))
    out = {"impl": impl, "losses": losses, "seconds": time.time() - t0, "opt_seed": opt_seed,
           "state_layout": state_layout(opt, model), "init_state": init_state}
    if ranks:
        out["mean_ranks"] = ranks
    return out


def compare(ours: List[float], ref: List[float], spread: List[float] = None) -> Dict:
    n = min(len(ours), len(ref))
    diffs = [abs(x - y) for x, y in zip(ours[:n], ref[:n])]
    tail = max(1, n // 5)
    out = {"max_abs_diff": max(diffs), "mean_abs_diff": sum(diffs) / n,
           "final_ours": ours[n - 1], "final_ref": ref[n - 1],
           "tail_mean_ours": sum(ours[n - tail:n]) / tail, "tail_mean_ref": sum(ref[n - tail:n]) / tail}
    out["tail_rel_diff"] = abs(out["tail_mean_ours"] - out["tail_mean_ref"]) / abs(out["tail_mean_ref"])
    if spread:
        out["ref_seed_spread_max_abs"] = max(spread)
    return out


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--preset", default="tiny")
    p.add_argument("--optimizer", choices=["dion", "muon", "adadion_v2"] + sorted(_LOWRANK), default="dion",
                   help="adadion_v2: adaptive rank, Q at --rank-fraction, starting at --init-rank-fraction; "
                        "the AdaDion family: --init-rank, --rank-min, --rank-max")
    p.add_argument("--impl", choices=["ours", "reference", "both"], default="both")
    p.add_argument("--device", default="cpu")
    p.add_argument("--dtype", choices=["fp32", "bf16", "mixed"], default="fp32")
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=0)
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--seq-len", type=int, default=256)
    p.add_argument("--data", choices=["fixed", "stream", "markov"], default="fixed")
    p.add_argument("--seed", type=int, default=0, help="model initialisation seed")
    p.add_argument("--data-seed", type=int, default=0)
    p.add_argument("--init", choices=["normal", "torchtitan"], default="normal")
    p.add_argument("--lr", type=float, default=0.01)
    p.add_argument("--mu", type=float, default=0.95)
    p.add_argument("--wd", type=float, default=0.0)
    p.add_argument("--rank-fraction", type=float, default=0.25)
    p.add_argument("--init-rank-fraction", type=float, default=0.125)
    p.add_argument("--rank-min", type=int, default=8)
    p.add_argument("--init-rank", type=int, default=32)
    p.add_argument("--rank-max", type=int, default=64)
    p.add_argument("--scalar-lr", type=float, default=3e-4)
    p.add_argument("--scalar-wd", type=float, default=0.1)
    p.add_argument("--ref-seeds", type=int, default=1, help="reference runs with optimizer seeds 0..n-1")
    p.add_argument("--out", default="")
    p.add_argument("--golden", default="", help="also write the compact golden file used by the tests")
    return p.parse_args(argv)


def golden_record(res: Dict) -> Dict:
    """The compact form committed as a golden file: the run's configuration,
    the reference's loss curves (every optimizer seed), this package's curve
    and the reference's optimizer-state layout."""
    ref = res["reference"]
    rec = {"config": res["config"],
           "reference_losses": [ref["losses"]] + [o["losses"] for o in res.get("reference_other_seeds", [])],
           "ours_losses": res["ours"]["losses"],
           "reference_state_layout": ref["state_layout"],
           "comparison": res.get("comparison")}
    if "mean_ranks" in ref:
        rec["reference_mean_ranks"] = [ref["mean_ranks"]] + [o["mean_ranks"]
                                                              for o in res.get("reference_other_seeds", [])]
        rec["ours_mean_ranks"] = res["ours"].get("mean_ranks")
    rec["config"].pop("golden", None)
    return rec


def main(argv=None) -> Dict:
    a = parse(argv)
    res: Dict = {"config": {k: v for k, v in vars(a).items() if k not in ("out", "golden")}}
    init_state = None
    if a.impl in ("ours", "both"):
        r = run_arm("ours", a)
        init_state = r.pop("init_state")
        res["ours"] = r
        print(json.dumps({"arm": "ours", "final": r["losses"][-1], "s": r["seconds"]}), flush=True)
    if a.impl in ("reference", "both"):
        if not os.path.isdir(os.path.join(REF_PATH, "ada_dion")):
            res["reference"] = {"unavailable": "baseline/_ref not installed"}
        else:
            runs = []
            for s in range(a.ref_seeds):
                r = run_arm("reference", a, init_state=init_state, opt_seed=s)
                r.pop("init_state")
                runs.append(r)
                print(json.dumps({"arm": f"reference[seed {s}]", "final": r["losses"][-1], "s": r["seconds"]}),
                      flush=True)
            res["reference"] = runs[0]
            if len(runs) > 1:
                res["reference_other_seeds"] = runs[1:]
    if "ours" in res and isinstance(res.get("reference"), dict) and "losses" in res["reference"]:
        spread = None
        if res.get("reference_other_seeds"):
            r0 = res["reference"]["losses"]
            spread = [max(abs(x - y) for x, y in zip(r0, o["losses"])) for o in res["reference_other_seeds"]]
        res["comparison"] = compare(res["ours"]["losses"], res["reference"]["losses"], spread)
        print(json.dumps({"comparison": res["comparison"]}), flush=True)
    if a.out:
        with open(a.out, "w") as fh:
            json.dump(res, fh, indent=1)
    if a.golden and "comparison" in res:
        with open(a.golden, "w") as fh:
            json.dump(golden_record(res), fh)
    return res


if __name__ == "__main__":
    main()
