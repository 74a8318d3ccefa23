"""Pipeline parallelism for the Llama model over NCCL point-to-point.

``build_pipeline_stage`` keeps this rank's contiguous share of transformer
blocks (plus the embedding on the first stage and the final norm + LM head
on the last), and ``PipelineRunner`` drives ``torch.distributed.pipelining``
(GPipe or 1F1B) over micro-batches: activations and their gradients move
between stages with NCCL send/recv, overlapped with the neighbours' compute
by the schedule. The loss on the last stage is the package's chunked
LM-head cross-entropy, so full logits are never materialised.

The reference registers ``pipelining_fn=pipeline_llm`` for its Llama specs
(ada_dion/integration/config_registry.py:99,150) without enabling it; its
optimizer container already keeps one optimizer per model part, which is
what a pipeline stage is here too.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from ..models import layers as L

__all__ = ["PipelineStageModule", "build_pipeline_stage", "PipelineRunner", "stage_layer_range"]


def stage_layer_range(n_layers: int, stage: int, n_stages: int) -> Tuple[int, int]:
    """Contiguous block range [lo, hi) of ``stage`` (earlier stages take the remainder)."""
    base, rem = divmod(n_layers, n_stages)
    lo = stage * base + min(stage, rem)
    return lo, lo + base + (1 if stage < rem else 0)


class PipelineStageModule(nn.Module):
    """One pipeline stage of a :class:`~dion_b200.models.llama3.Transformer`.
    Parameter names keep the full model's FQNs (``layers.<i>...``), so
    checkpoints and optimizer groups are unchanged."""

    def __init__(self, model: nn.Module, stage: int, n_stages: int):
        super().__init__()
        self.cfg = model.cfg
        self.first, self.last = stage == 0, stage == n_stages - 1
        lo, hi = stage_layer_range(model.cfg.n_layers, stage, n_stages)
        self.tok_embeddings = model.tok_embeddings if self.first else None
        self.layers = nn.ModuleDict({str(i): model.layers[str(i)] for i in range(lo, hi)})
        self.norm = model.norm if self.last else None
        self.output = model.output if self.last else None
        self.register_buffer("rope_cache", model.rope_cache, persistent=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = self.tok_embeddings(x) if self.first else x
        rope = self.rope_cache[: h.shape[1]].float()
        for layer in self.layers.values():
            h = layer(h, rope)
        if self.last:
            h = self.norm(h)
        return h

    def loss(self, h: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        return L.linear_cross_entropy(h, self.output.weight, labels)


def build_pipeline_stage(model: nn.Module, pp_mesh) -> PipelineStageModule:
    return PipelineStageModule(model, pp_mesh.get_local_rank(), pp_mesh.size())


class PipelineRunner:
    """Runs one optimisation step's forward/backward through the pipeline."""

    def __init__(self, stage_module: PipelineStageModule, pp_mesh, device: torch.device, n_microbatches: int,
                 schedule: str = "1F1B"):
        from torch.distributed.pipelining import PipelineStage, Schedule1F1B, ScheduleGPipe

        self.module = stage_module
        self.pp_group = pp_mesh.get_group()
        self.pp_rank, self.pp_size = pp_mesh.get_local_rank(), pp_mesh.size()
        self.stage = PipelineStage(stage_module, self.pp_rank, self.pp_size, device, group=self.pp_group)
        cls = {"1F1B": Schedule1F1B, "GPipe": ScheduleGPipe}[schedule]
        self.schedule = cls(self.stage, n_microbatches=n_microbatches, loss_fn=self._loss, scale_grads=True)
        self.device = device

    def _loss(self, h: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        return self.module.loss(h, labels)

    def step(self, tokens: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        """Forward + backward of a whole batch; returns the mean loss on every stage."""
        losses: List[torch.Tensor] = []
        if self.pp_rank == 0:
            self.schedule.step(tokens)
        elif self.pp_rank == self.pp_size - 1:
            self.schedule.step(target=labels, losses=losses)
        else:
            self.schedule.step()
        return self._broadcast_loss(losses)

    def _broadcast_loss(self, losses: List[torch.Tensor]) -> torch.Tensor:
        loss = torch.stack(losses).mean().detach() if losses else torch.zeros((), device=self.device)
        # the loss lives on the last stage; every stage reports it
        dist.broadcast(loss, group_src=self.pp_size - 1, group=self.pp_group)
        return loss

    @torch.no_grad()
    def eval(self, tokens: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        """Forward only (the schedule's evaluation pass, no gradients); returns
        the mean loss on every stage."""
        losses: List[torch.Tensor] = []
        if self.pp_rank == 0:
            self.schedule.eval(tokens)
        elif self.pp_rank == self.pp_size - 1:
            self.schedule.eval(target=labels, losses=losses)
        else:
            self.schedule.eval()
        return self._broadcast_loss(losses)
