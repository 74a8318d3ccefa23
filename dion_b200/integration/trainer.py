"""Minimal Llama trainer (no torchtitan needed).

One process per GPU; FSDP2/HSDP over the data-parallel mesh; the hybrid
optimizer container; warmup + cosine LR schedule with a floor (as in
ada_dion/integration/config_registry.py:161-184: warmup 200, cosine decay
to 10 %, grad-norm clip 1.0); synthetic uniform tokens or token files read
by the native loader (:mod:`dion_b200.data`), with an optional validation
pass over held-out token files.

``train_step`` is the public per-step API: it takes the step's host batch
(pinned int64 tokens / labels), copies it to the device, runs forward,
backward, clipping and the optimizer, and returns the loss tensor.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from ..data import SyntheticTokens, TokenFileLoader, build_loader  # noqa: F401 (re-exported)
from ..models.llama3 import Llama3Config, Transformer, llama3_config
from ..parallel.fsdp import apply_fsdp
from ..parallel.tp import apply_tp
from ..parallel.mesh import ParallelDims, build_mesh, init_distributed
from .hybrid_optimizer import HybridOptimizersContainer

__all__ = ["TrainerConfig", "Trainer", "SyntheticTokens", "lr_lambda"]


@dataclass
class TrainerConfig:
    model: str = "1B"
    model_overrides: Dict = field(default_factory=dict)
    seq_len: int = 4096
    local_batch_size: int = 8
    steps: int = 100
    warmup_steps: int = 200
    decay_ratio: Optional[float] = None
    decay_type: str = "cosine"
    min_lr_factor: float = 0.1
    max_norm: float = 1.0
    seed: int = 2
    init_mode: str = "normal"
    dp_replicate: int = 1
    dp_shard: int = -1
    tp: int = 1
    pp: int = 1
    pp_microbatches: int = 0  # 0: 2 x pp
    pp_schedule: str = "1F1B"  # 1F1B | GPipe
    use_fsdp: bool = True
    ac_mode: str = "none"  # none | full | selective
    ac_option: str = "op"
    # with tp > 1: token-sharded activations between sublayers and the TP
    # collectives fused into the GEMMs (parallel/sp.py); False: plain TP
    sequence_parallel: bool = True
    optimizer: HybridOptimizersContainer.Config = field(default_factory=HybridOptimizersContainer.Config)
    log_freq: int = 10
    # "synthetic", or token files (comma-separated files, directories of *.bin, globs)
    dataset: str = "synthetic"
    data_shuffle: bool = True
    data_prefetch: int = 4
    data_bytes_per_token: int = 0  # raw token files only (files with a header carry it)
    data_tokenizer: str = "byte"  # "text:<files>" datasets: "byte" or a local HuggingFace tokenizer directory
    data_text_field: str = "text"
    # held-out token files for ``validate`` ("" = none)
    val_dataset: str = ""
    # sequences per optimizer step over all data-parallel ranks; a multiple of
    # local_batch_size x the data-parallel degree, the quotient being the number
    # of accumulated micro-batches (-1: no accumulation)
    global_batch_size: int = -1
    # FSDP mixed precision: dtype of the gathered parameters (compute) and of
    # the gradient reduction
    param_dtype: str = "bfloat16"
    reduce_dtype: str = "float32"


def lr_lambda(step: int, warmup: int, total: int, min_factor: float, decay_ratio: Optional[float] = None,
              decay_type: str = "cosine") -> float:
    """Multiplier on the base lr: linear warm-up over ``warmup`` steps, an
    optional stable phase, then decay to ``min_factor`` over the last
    ``decay_ratio * total`` steps (all the steps after warm-up when
    ``decay_ratio`` is None), shaped ``cosine``, ``linear`` or ``sqrt``
    (1 - sqrt(progress)): torchtitan's warmup-stable-decay schedule, which
    the reference configures (ada_dion/integration/config_registry.py:171-176)."""
    if warmup > 0 and step < warmup:
        return (step + 1) / (warmup + 1)
    decay = total - warmup if decay_ratio is None else int(round(total * decay_ratio))
    decay = max(0, min(decay, total - warmup))
    start = total - decay
    if step < start or decay <= 0:
        return 1.0
    prog = min(1.0, (step - start) / max(1, decay))
    if decay_type == "linear":
        adj = 1.0 - prog
    elif decay_type == "sqrt":
        adj = 1.0 - math.sqrt(prog)
    elif decay_type == "cosine":
        adj = 0.5 * (1 + math.cos(math.pi * prog))
    else:
        raise ValueError(f"decay_type must be cosine, linear or sqrt, got {decay_type!r}")
    return min_factor + (1 - min_factor) * adj


def clip_grad_norm_multi_mesh_(params: List[torch.nn.Parameter], max_norm: float,
                               stage_group=None) -> torch.Tensor:
    """Global-norm clipping when gradients live on different meshes (FSDP-only
    and FSDP x TP DTensors in one model): norms are taken per (mesh,
    placements) group, made replicated, and combined; the clip coefficient
    scales every local shard. ``stage_group``: the pipeline group, whose
    stages hold disjoint parameters (their squared norms are summed)."""
    from torch.distributed.tensor import DTensor

    groups: Dict[Any, List[torch.Tensor]] = {}
    for p in params:
        g = p.grad
        if g is None:
            continue
        key = (id(g.device_mesh), tuple(g.placements)) if isinstance(g, DTensor) else None
        groups.setdefault(key, []).append(g)
    sq = []
    for gs in groups.values():
        n = torch.nn.utils.get_total_norm(gs, 2.0, foreach=True)
        if isinstance(n, DTensor):
            n = n.full_tensor()
        sq.append(n.float().square())
    total_sq = torch.stack(sq).sum() if sq else torch.zeros((), device=params[0].device)
    if stage_group is not None:
        dist.all_reduce(total_sq, group=stage_group)
    total = total_sq.sqrt()
    coef = (max_norm / (total + 1e-6)).clamp(max=1.0)
    for gs in groups.values():
        torch._foreach_mul_([g.to_local() if isinstance(g, DTensor) else g for g in gs], coef)
    return total


class Trainer:
    def __init__(self, cfg: TrainerConfig, device: Optional[torch.device] = None):
        self.cfg = cfg
        self.rank, self.world, self.local_rank = init_distributed()
        if device is None:
            device = torch.device("cuda", self.local_rank) if torch.cuda.is_available() else torch.device("cpu")
        self.device = device
        self.mesh = None
        shard_mesh = replicate_mesh = None
        dims = ParallelDims(cfg.dp_replicate, cfg.dp_shard, cfg.tp, cfg.pp)
        self.dp_mesh = None
        if not cfg.use_fsdp and self.world // (max(1, cfg.tp) * max(1, cfg.pp)) > 1:
            # without FSDP nothing would reduce gradients across data-parallel ranks
            raise ValueError("use_fsdp=False needs a single data-parallel rank; for replicated data "
                             "parallelism keep FSDP and set dp_replicate (HSDP with dp_shard=1)")
        if cfg.use_fsdp or cfg.pp > 1:
            self.mesh = build_mesh(dims, device.type)
            names = self.mesh.mesh_dim_names
            dp_names = tuple(n for n in ("dp_replicate", "dp_shard") if n in names)
            if dp_names:
                self.dp_mesh = self.mesh[dp_names] if len(dp_names) > 1 else self.mesh[dp_names[0]]
            shard_mesh = self.mesh["dp_shard"] if "dp_shard" in names else None
            replicate_mesh = self.mesh["dp_replicate"] if "dp_replicate" in names else None
        mcfg: Llama3Config = llama3_config(cfg.model, **cfg.model_overrides)
        mcfg.max_seq_len = max(mcfg.max_seq_len, cfg.seq_len)
        self.model_cfg = mcfg
        torch.manual_seed(cfg.seed)
        with torch.device(device):
            model = Transformer(mcfg)
        gen = torch.Generator(device=device).manual_seed(cfg.seed)
        model.init_weights(cfg.init_mode, generator=gen)
        model.set_activation_checkpointing(cfg.ac_mode, cfg.ac_option)
        self.pp_runner = None
        self.pp_group = None
        if cfg.pp > 1:
            from ..parallel.pp import PipelineRunner, build_pipeline_stage

            pp_mesh = self.mesh["pp"]
            model = build_pipeline_stage(model, pp_mesh)
            self.pp_group = pp_mesh.get_group()
        tp_mesh = None
        if cfg.tp > 1:
            if self.mesh is None or "tp" not in self.mesh.mesh_dim_names:
                raise ValueError("tensor parallelism needs use_fsdp=True (the mesh is built there)")
            tp_mesh = self.mesh["tp"]
            apply_tp(model, tp_mesh, sequence_parallel=cfg.sequence_parallel and cfg.pp == 1)
        if cfg.use_fsdp and self.dp_mesh is not None:
            # pipeline stages keep their parameters gathered across micro-batches
            # (and the last stage's LM head stays gathered for the loss)
            apply_fsdp(model, self.dp_mesh, param_dtype=getattr(torch, cfg.param_dtype),
                       reduce_dtype=getattr(torch, cfg.reduce_dtype), reshard_after_forward=cfg.pp == 1)
        if cfg.pp > 1:
            self.pp_runner = PipelineRunner(model, self.mesh["pp"], device, cfg.pp_microbatches or 2 * cfg.pp,
                                            cfg.pp_schedule)
        self.model = model
        self.tp_mesh = tp_mesh
        self.optimizers = HybridOptimizersContainer(
            cfg.optimizer, model_parts=[model], shard_mesh=shard_mesh, replicate_mesh=replicate_mesh, tp_mesh=tp_mesh
        )
        self._base_lrs = [[g["lr"] for g in o.param_groups] for o in self.optimizers]
        self.step_idx = 0
        # mesh order (pp, dp_replicate, dp_shard, tp): the ranks of one TP group
        # and of one pipeline share a batch
        tp, pp = max(1, cfg.tp), max(1, cfg.pp)
        per_stage = self.world // pp
        self.data_rank, self.data_world = (self.rank % per_stage) // tp, per_stage // tp
        self.grad_accum = 1
        if cfg.global_batch_size and cfg.global_batch_size > 0:
            per_pass = cfg.local_batch_size * self.data_world
            if cfg.global_batch_size % per_pass:
                raise ValueError(f"global_batch_size {cfg.global_batch_size} is not a multiple of local_batch_size x "
                                 f"data-parallel degree = {per_pass}")
            self.grad_accum = cfg.global_batch_size // per_pass
            if self.grad_accum > 1 and cfg.pp > 1:
                raise ValueError("with pipeline parallelism set pp_microbatches instead of gradient accumulation")
        # each step reads grad_accum micro-batches of local_batch_size sequences
        self.data = build_loader(cfg.dataset, vocab=mcfg.vocab_size, seq_len=cfg.seq_len,
                                 local_batch=cfg.local_batch_size * self.grad_accum, seed=cfg.seed, rank=self.data_rank,
                                 world=self.data_world, shuffle=cfg.data_shuffle, prefetch=cfg.data_prefetch,
                                 bytes_per_token=cfg.data_bytes_per_token, tokenizer=cfg.data_tokenizer,
                                 text_field=cfg.data_text_field)
        self.val_data = None
        if cfg.val_dataset:  # token files or "text:<files>", read in order from the start on every pass
            self.val_data = build_loader(cfg.val_dataset, vocab=mcfg.vocab_size, seq_len=cfg.seq_len,
                                         local_batch=cfg.local_batch_size, seed=cfg.seed, rank=self.data_rank,
                                         world=self.data_world, shuffle=False, prefetch=cfg.data_prefetch,
                                         bytes_per_token=cfg.data_bytes_per_token, tokenizer=cfg.data_tokenizer,
                                         text_field=cfg.data_text_field)

    @property
    def last_grad_norm(self) -> float:
        gn = getattr(self, "_grad_norm", None)
        if gn is None:
            return float("nan")
        gn = gn.full_tensor() if hasattr(gn, "full_tensor") else gn
        return float(gn)

    def _set_lr(self) -> None:
        c = self.cfg
        total = c.steps
        f = lr_lambda(self.step_idx, c.warmup_steps, total, c.min_lr_factor, c.decay_ratio, c.decay_type)
        for opt, base in zip(self.optimizers, self._base_lrs):
            for g, b in zip(opt.param_groups, base):
                g["lr"] = b * f

    def forward_backward(self, tokens: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        loss = self.model.loss(tokens, labels)
        loss.backward()
        sp = getattr(self.model, "sp", None)
        if sp is not None:
            # each TP rank back-propagated its own tokens: sum the shared parameters'
            # gradients, and report the whole batch's loss
            from ..parallel.tp import sp_sync_replicated_grads

            sp_sync_replicated_grads(self.model, sp.group)
            loss = loss.detach().clone()
            torch.distributed.all_reduce(loss, group=sp.group)
        return loss

    def _accumulate(self, tokens: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        """Gradient accumulation: the step's rows as ``grad_accum`` micro-batches
        (FSDP reduce-scatters each micro-batch's gradients into the sharded
        accumulators), each loss scaled by 1 / grad_accum; the TP sum of
        replicated parameters' gradients runs once, after the last. Returns
        the step's mean loss."""
        n = self.grad_accum
        total = None
        for t, l in zip(tokens.chunk(n), labels.chunk(n)):
            loss = self.model.loss(t, l)
            (loss / n).backward()
            d = loss.detach() / n
            total = d if total is None else total + d
        sp = getattr(self.model, "sp", None)
        if sp is not None:
            from ..parallel.tp import sp_sync_replicated_grads

            sp_sync_replicated_grads(self.model, sp.group)
            total = total.clone()
            torch.distributed.all_reduce(total, group=sp.group)
        return total

    def train_step(self, tokens: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        """One optimisation step on a host (or device) batch; returns the device loss."""
        tokens = tokens.to(self.device, non_blocking=True)
        labels = labels.to(self.device, non_blocking=True)
        self._set_lr()
        if self.pp_runner is not None:
            loss = self.pp_runner.step(tokens, labels)
        elif self.grad_accum > 1:
            loss = self._accumulate(tokens, labels)
        else:
            loss = self.forward_backward(tokens, labels)
        if self.cfg.max_norm and self.cfg.max_norm > 0:
            if self.tp_mesh is not None or self.pp_group is not None:
                self._grad_norm = clip_grad_norm_multi_mesh_(list(self.model.parameters()), self.cfg.max_norm,
                                                             self.pp_group)
            else:
                self._grad_norm = torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.cfg.max_norm,
                                                                 foreach=True)
        self.optimizers.step()
        self.optimizers.zero_grad(set_to_none=True)
        self.step_idx += 1
        return loss.detach()

    @torch.no_grad()
    def validate(self, steps: int) -> float:
        """Mean loss over the first ``steps`` batches of the validation files
        (read from their start on every call, in file order), averaged over
        the data-parallel ranks; the same value is returned on every rank."""
        if self.val_data is None:
            raise ValueError("no validation dataset configured (TrainerConfig.val_dataset)")
        self.val_data.load_state_dict({"samples": 0})
        total = torch.zeros((), device=self.device, dtype=torch.float32)
        for _ in range(steps):
            t, l = self.val_data.next()
            t, l = t.to(self.device, non_blocking=True), l.to(self.device, non_blocking=True)
            if self.pp_runner is not None:  # the schedule's forward-only pass; every stage gets the loss
                total += self.pp_runner.eval(t, l).float()
                continue
            loss = self.model.loss(t, l)
            sp = getattr(self.model, "sp", None)
            if sp is not None:  # each TP rank holds its tokens' share of the batch loss
                loss = loss.detach().clone()
                dist.all_reduce(loss, group=sp.group)
            total += loss.float()
        total /= max(1, steps)
        if dist.is_initialized() and dist.get_world_size() > 1:
            # TP ranks hold equal values: the sum over all ranks / world = mean over DP ranks
            dist.all_reduce(total)
            total /= dist.get_world_size()
        return float(total)

    def train(self, steps: Optional[int] = None, log=print) -> List[float]:
        steps = steps or self.cfg.steps
        losses = []
        t0 = time.perf_counter()
        for i in range(steps):
            t, l = self.data.next()
            loss = self.train_step(t, l)
            if (i + 1) % self.cfg.log_freq == 0 or i == steps - 1:
                v = loss.item()
                losses.append(v)
                if self.rank == 0 and log:
                    dt = time.perf_counter() - t0
                    log(f"step {self.step_idx} loss {v:.4f} ({dt:.1f}s)")
        return losses
