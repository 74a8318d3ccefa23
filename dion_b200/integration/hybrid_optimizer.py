"""HybridOptimizersContainer: one optimizer per model part covering the
matrix group (Muon / Dion / Dion2 / AdaDion variants) and the AdamW scalar
groups (embeddings, LM head at lr/sqrt(d_model), norms without weight decay).

Behaviour follows ada_dion/integration/hybrid_optimizer.py:51-317 (Config
fields, group construction, DCP-flattened ``state_dict``), with two
deliberate differences:
  * it does not need torchtitan: it is a plain container usable by the
    package's own trainer (and by torchtitan, which only iterates it);
  * it passes the real FSDP shard sub-mesh (and the replicate mesh, for Dion)
    instead of a fresh 1-D world mesh, so HSDP works.
"""
from __future__ import annotations

import functools
import math
from dataclasses import dataclass, field, fields
from typing import Any, Dict, Iterator, List, Optional

import torch
import torch.nn as nn
from torch.distributed.checkpoint.state_dict import StateDictOptions, get_optimizer_state_dict, set_optimizer_state_dict
from torch.distributed.device_mesh import DeviceMesh
from torch.optim import Optimizer

from .param_grouper import group_params_for_hybrid

__all__ = ["HybridOptimizersContainer", "build_param_groups"]


def build_param_groups(model: nn.Module, cfg: "HybridOptimizersContainer.Config") -> List[Dict[str, Any]]:
    g = group_params_for_hybrid(model)
    groups: List[Dict[str, Any]] = []
    scalar = dict(
        algorithm=cfg.scalar_algorithm,
        beta1=cfg.scalar_beta1,
        beta2=cfg.scalar_beta2,
        epsilon=cfg.scalar_eps,
    )
    if g.matrix_params:
        groups.append({"params": g.matrix_params})
    if g.embed_params:
        groups.append({"params": g.embed_params, "lr": cfg.scalar_lr, "weight_decay": cfg.scalar_weight_decay, **scalar})
    if g.output_params:
        d_model = g.output_params[0].shape[-1]
        groups.append(
            {
                "params": g.output_params,
                "lr": cfg.scalar_lr / math.sqrt(d_model) if cfg.output_head_lr_scaling else cfg.scalar_lr,
                "weight_decay": cfg.scalar_weight_decay,
                **scalar,
            }
        )
    if g.norm_params:
        groups.append({"params": g.norm_params, "lr": cfg.scalar_lr, "weight_decay": 0.0, **scalar})
    return groups


class HybridOptimizersContainer(Optimizer):
    @dataclass
    class Config:
        name: str = "Muon"
        lr: float = 0.02
        weight_decay: float = 0.01
        # Muon
        mu: float = 0.95
        nesterov: bool = False
        adjust_lr: Optional[str] = "spectral_norm"
        ns_coeffs: Any = None
        # Dion
        rank_fraction: float = 0.25
        power_iters: int = 1
        # Dion2
        fraction: float = 0.25
        ef_decay: float = 0.95
        # AdaDion (routed to SDion modes, as in the reference container)
        init_rank: int = 64
        adaptive_rank: bool = True
        erank_ema_beta: float = 0.9
        rho: float = 1.5
        rank_min: int = 16
        rank_max: int = 256
        rank_quantize: int = 8
        rank_warmup_steps: int = 10
        warmup_rank: int = 128
        rank_step_up: int = 16
        rank_step_down: int = 8
        use_quality_control: bool = True
        aerr_ema_beta: float = 0.95
        aerr_target: float = 0.08
        aerr_up_margin: float = 0.15
        aerr_down_margin: float = 0.15
        use_anchor: bool = True
        anchor_alpha: float = 0.1
        anchor_period: int = 50
        sdion_mode: str = "baseline"
        qbuf_max_cols: int = 256
        # --- Dion2 row selection: "top_l1" or "random" ---
        selection_method: str = "top_l1"
        # --- GSDion switches ---
        rank_normalize: bool = True
        use_adaptive_scalar: bool = True
        use_rms_matching: bool = True
        use_trust_region: bool = True
        use_residual_rank: bool = True
        # AdaDionV2 (adaptive-rank Dion)
        rank_fraction_max: float = 0.7
        init_rank_fraction: float = 0.25
        rank_scale: float = 1.5
        # LM head lr = scalar_lr / sqrt(d_model) (the reference container's rule); False: scalar_lr
        output_head_lr_scaling: bool = True
        # scalar groups
        scalar_algorithm: str = "adamw"
        scalar_lr: float = 3e-4
        scalar_weight_decay: float = 0.01
        scalar_beta1: float = 0.95
        scalar_beta2: float = 0.95
        scalar_eps: float = 1e-8

    def __init__(
        self,
        config: "HybridOptimizersContainer.Config",
        *,
        model_parts: List[nn.Module],
        shard_mesh: Optional[DeviceMesh] = None,
        replicate_mesh: Optional[DeviceMesh] = None,
        tp_mesh: Optional[DeviceMesh] = None,
    ) -> None:
        self.config = config
        self.model_parts = model_parts
        self.optimizers: List[Optimizer] = []
        all_params: List[nn.Parameter] = []
        for model in model_parts:
            groups = build_param_groups(model, config)
            opt = self._create_optimizer(config, groups, shard_mesh, replicate_mesh, tp_mesh)
            self.optimizers.append(opt)
            for g in groups:
                all_params.extend(g["params"])
        Optimizer.__init__(self, all_params, {"lr": config.lr})

    @staticmethod
    def _create_optimizer(cfg, groups, shard_mesh, replicate_mesh, tp_mesh) -> Optimizer:
        from .. import optim

        name = cfg.name
        if name == "AdamW":
            # every group on the scalar rule; the matrix group takes the main lr / wd
            for g in groups:
                g.setdefault("lr", cfg.lr)
                g.setdefault("weight_decay", cfg.weight_decay)
                g.update(algorithm="adamw", beta1=cfg.scalar_beta1, beta2=cfg.scalar_beta2, epsilon=cfg.scalar_eps)
            return optim.Muon(groups, distributed_mesh=shard_mesh, lr=cfg.lr, weight_decay=cfg.weight_decay)
        if name == "Muon":
            Muon = optim.Muon
            return Muon(groups, distributed_mesh=shard_mesh, lr=cfg.lr, mu=cfg.mu, weight_decay=cfg.weight_decay,
                        nesterov=cfg.nesterov, adjust_lr=cfg.adjust_lr, ns_coeffs=cfg.ns_coeffs, tp_mesh=tp_mesh)
        if name == "Dion":
            return optim.Dion(groups, replicate_mesh=replicate_mesh, outer_shard_mesh=shard_mesh, inner_shard_mesh=tp_mesh,
                        lr=cfg.lr, mu=cfg.mu, rank_fraction=cfg.rank_fraction, weight_decay=cfg.weight_decay)
        if name == "Dion2":
            return optim.Dion2(groups, distributed_mesh=shard_mesh, lr=cfg.lr, fraction=cfg.fraction,
                         ef_decay=cfg.ef_decay, weight_decay=cfg.weight_decay, tp_mesh=tp_mesh,
                         selection_method=cfg.selection_method)
        if name == "AdaDionV2":
            return optim.AdaDionV2(groups, replicate_mesh=replicate_mesh, outer_shard_mesh=shard_mesh,
                             inner_shard_mesh=tp_mesh, lr=cfg.lr, mu=cfg.mu, weight_decay=cfg.weight_decay,
                             # Q width: rank_fraction_max with adaptive rank, rank_fraction without
                             # (ada_dion/optim/config_registry.py:72)
                             rank_fraction_max=cfg.rank_fraction_max if cfg.adaptive_rank else cfg.rank_fraction,
                             adaptive_rank=cfg.adaptive_rank, init_rank_fraction=cfg.init_rank_fraction,
                             rank_min=cfg.rank_min, rank_quantize=cfg.rank_quantize, rank_step_up=cfg.rank_step_up,
                             rank_step_down=cfg.rank_step_down, erank_ema_beta=cfg.erank_ema_beta,
                             rank_scale=cfg.rank_scale)
        if name == "AdaDion":
            if tp_mesh is not None:
                raise ValueError("AdaDion (SDion) supports data-parallel layouts (DDP / FSDP); it has no "
                                 "tensor-parallel path")
            mode_kw = {
                "baseline": dict(enable_skip=False, enable_consensus=False, enable_anchor=False, enable_recovery=False),
                "skip": dict(enable_skip=True, enable_consensus=False, enable_anchor=False, enable_recovery=True),
                "skip_consensus": dict(enable_skip=True, enable_consensus=True, enable_anchor=False, enable_recovery=True),
                "skip_cons_anchor": dict(enable_skip=True, enable_consensus=True, enable_anchor=True, enable_recovery=True),
            }.get(cfg.sdion_mode, {})
            return optim.SDion(groups, device_mesh=shard_mesh, lr=cfg.lr, mu=cfg.mu, init_rank=cfg.init_rank,
                         rank_min=cfg.rank_min, rank_max=cfg.rank_max, qbuf_max_cols=cfg.qbuf_max_cols,
                         weight_decay=cfg.weight_decay, **mode_kw)
        # the research variants by class name (the reference container reaches only SDion, as "AdaDion")
        if tp_mesh is not None and name in ("AdaDionAnchor", "SDion", "GSDion", "AGDion", "QCDion"):
            raise ValueError(f"{name} supports data-parallel layouts (DDP / FSDP); it has no tensor-parallel path")
        lowrank = dict(device_mesh=shard_mesh, lr=cfg.lr, mu=cfg.mu, init_rank=cfg.init_rank, rank_min=cfg.rank_min,
                       rank_max=cfg.rank_max, qbuf_max_cols=cfg.qbuf_max_cols, weight_decay=cfg.weight_decay)
        if name == "AdaDionAnchor":  # the plain AdaDion class (ANCHOR-MBP)
            return optim.AdaDion(groups, adaptive_rank=cfg.adaptive_rank, erank_ema_beta=cfg.erank_ema_beta,
                                 rho=cfg.rho, rank_quantize=cfg.rank_quantize, rank_warmup_steps=cfg.rank_warmup_steps,
                                 warmup_rank=cfg.warmup_rank, rank_step_up=cfg.rank_step_up,
                                 rank_step_down=cfg.rank_step_down, use_quality_control=cfg.use_quality_control,
                                 aerr_ema_beta=cfg.aerr_ema_beta, aerr_target=cfg.aerr_target,
                                 aerr_up_margin=cfg.aerr_up_margin, aerr_down_margin=cfg.aerr_down_margin,
                                 use_anchor=cfg.use_anchor, anchor_alpha=cfg.anchor_alpha,
                                 anchor_period=cfg.anchor_period, **lowrank)
        if name == "SDion":
            return optim.SDion(groups, **lowrank)
        if name == "GSDion":
            return optim.GSDion(groups, use_anchor=cfg.use_anchor, anchor_alpha=cfg.anchor_alpha,
                                anchor_period=cfg.anchor_period, rank_normalize=cfg.rank_normalize,
                                use_adaptive_scalar=cfg.use_adaptive_scalar, use_rms_matching=cfg.use_rms_matching,
                                use_trust_region=cfg.use_trust_region, use_residual_rank=cfg.use_residual_rank,
                                **lowrank)
        if name == "AGDion":
            return optim.AGDion(groups, use_anchor=cfg.use_anchor, anchor_alpha=cfg.anchor_alpha, **lowrank)
        if name == "QCDion":
            return optim.QCDion(groups, **lowrank)
        raise ValueError(f"Unknown matrix optimizer: {name!r}. Supported: 'AdamW', 'Muon', 'Dion', 'Dion2', 'AdaDion', "
                         "'AdaDionV2', 'AdaDionAnchor', 'SDion', 'GSDion', 'AGDion', 'QCDion'")

    def __iter__(self) -> Iterator[Optimizer]:
        return iter(self.optimizers)

    def __len__(self) -> int:
        return len(self.optimizers)

    def step(self, *args, **kwargs) -> None:
        for opt in self.optimizers:
            opt.step(*args, **kwargs)

    def zero_grad(self, *args, **kwargs) -> None:
        for opt in self.optimizers:
            opt.zero_grad(*args, **kwargs)

    def state_dict(self) -> Dict[str, Any]:
        """DCP-flattened optimizer state (``state.<fqn>.<key>``, ``param_groups.<fqn>.<hyper>``)."""
        fn = functools.partial(get_optimizer_state_dict, options=StateDictOptions(flatten_optimizer_state_dict=True))
        sd: Dict[str, Any] = {}
        for model, opt in zip(self.model_parts, self.optimizers):
            sd.update(fn(model, opt))
        return sd

    def load_state_dict(self, state_dict: Dict[str, Any]) -> None:
        fn = functools.partial(
            set_optimizer_state_dict,
            optim_state_dict=state_dict,
            options=StateDictOptions(flatten_optimizer_state_dict=True),
        )
        for model, opt in zip(self.model_parts, self.optimizers):
            fn(model, opt)

    def init_cache_state_dict(self) -> None:
        pass

    def get_optimizers(self) -> List[Optimizer]:
        return self.optimizers
