"""AdaDionV2: Dion with optional adaptive rank.

Without ``adaptive_rank`` it is exactly :class:`~dion_b200.optim.dion.Dion`
(with this class's defaults: ``rank_fraction_max=0.7``,
``weight_decay=0.1``). With it (ada_dion/optim/adadion_v2.py:82-249,
:750-779, :1115-1295, :1451-1530):
  * Q is kept at ``r_cap = rank_fraction_max * min(m, n)`` columns and each
    matrix uses its active rank ``r`` (initially ``init_rank_fraction``);
  * after each step the column norms of R (the singular-value proxies,
    all-reduced across shards) give the entropy effective rank, its EMA sets
    the desired rank ``round(rank_scale * erank_ema)``, clamped to
    [rank_min, r_cap], quantised to ``rank_quantize`` and rate-limited by
    ``rank_step_up`` / ``rank_step_down``; new Q columns are refilled with
    normalised Gaussians;
  * state adds ``r``, ``r_cap``, ``transpose``, ``erank_ema``, ``aerr_ema``
    and ``ada_step``; ``Q`` and ``momentum`` are plain local tensors.

Matrices of a shape group with different active ranks are still processed as
one batch: the GEMMs run at the group's largest active rank with the
inactive Q columns zeroed, and the orthogonalisation runs per distinct rank,
so no column beyond a matrix's rank enters its factorisation.
"""
from __future__ import annotations

import math
from typing import Any, Dict, List, Optional, Tuple, Union

import torch
from torch import Tensor
from torch.distributed import ProcessGroup
from torch.distributed.device_mesh import DeviceMesh
from torch.distributed.tensor import DTensor

from .. import ops
from ._utils import device_list, to_local
from .dion import Dion, DionMixedPrecisionConfig
from .linalg import orthogonalize

__all__ = ["AdaDionV2", "DionMixedPrecisionConfig"]


def _quantize_int(x: int, q: int) -> int:
    """Round x to the nearest multiple of q (at least q)."""
    if q <= 1:
        return x
    return max(q, q * round(x / q))


class AdaDionV2(Dion):
    def __init__(
        self,
        params,
        replicate_mesh: Optional[Union[DeviceMesh, ProcessGroup]] = None,
        outer_shard_mesh: Optional[DeviceMesh] = None,
        inner_shard_mesh: Optional[DeviceMesh] = None,
        replicate_mesh_grad_sync: bool = True,
        rank_fraction_max: float = 0.7,
        rank_multiple_of: int = 1,
        lr: float = 0.01,
        mu: float = 0.95,
        betas: Tuple[float, float] = (0.9, 0.95),
        weight_decay: float = 0.1,
        epsilon: float = 1e-8,
        power_iters: int = 1,
        qr_method: str = "rcqr",
        cqr_warmup_steps: int = 150,
        rcqr_oversample: float = 1.25,
        mixed_precision_config: Optional[DionMixedPrecisionConfig] = None,
        adaptive_rank: bool = False,
        init_rank_fraction: float = 0.25,
        erank_ema_beta: float = 0.9,
        rank_scale: float = 1.5,
        rank_min: int = 16,
        rank_quantize: int = 8,
        rank_step_up: int = 16,
        rank_step_down: int = 8,
        use_quality_control: bool = False,
        aerr_ema_beta: float = 0.95,
        aerr_target: float = 0.08,
        aerr_up_margin: float = 0.15,
        aerr_down_margin: float = 0.15,
        adapt_step: int = 1,
    ):
        if rank_fraction_max <= 0 or rank_fraction_max > 1:
            raise ValueError(f"Invalid rank_fraction_max: {rank_fraction_max}")
        super().__init__(
            params, replicate_mesh=replicate_mesh, outer_shard_mesh=outer_shard_mesh,
            inner_shard_mesh=inner_shard_mesh, replicate_mesh_grad_sync=replicate_mesh_grad_sync,
            rank_fraction=rank_fraction_max, rank_multiple_of=rank_multiple_of, lr=lr, mu=mu, betas=betas,
            weight_decay=weight_decay, epsilon=epsilon, power_iters=power_iters, qr_method=qr_method,
            cqr_warmup_steps=cqr_warmup_steps, rcqr_oversample=rcqr_oversample,
            mixed_precision_config=mixed_precision_config,
        )
        self._adaptive_rank = adaptive_rank
        self._ada_config = dict(
            init_rank_fraction=init_rank_fraction, erank_ema_beta=erank_ema_beta, rank_scale=rank_scale,
            rank_min=rank_min, rank_quantize=rank_quantize, rank_step_up=rank_step_up,
            rank_step_down=rank_step_down, use_quality_control=use_quality_control, aerr_ema_beta=aerr_ema_beta,
            aerr_target=aerr_target, aerr_up_margin=aerr_up_margin, aerr_down_margin=aerr_down_margin,
            adapt_step=adapt_step,
        )
        self._q_full: Dict[int, Tensor] = {}  # id(param) -> full-width Q slot (allocation width)

    # ------------------------------------------------------------------ state
    def _bind_arena(self, params, order, mom_arena, q_arena, cfg, q_shape) -> None:
        if not self._adaptive_rank or cfg.inner_shard_mesh_dim is not None:
            # matrices sharded over an inner (TP) mesh keep the fixed rank r_cap: the
            # FSDP x TP update takes no active rank (nor does the reference's,
            # ada_dion/optim/adadion_v2.py:1298-1448, which ignores r_list)
            return super()._bind_arena(params, order, mom_arena, q_arena, cfg, q_shape)
        key = tuple(id(p) for p in params)
        r_cap = q_shape[1]
        # allocation width rounded up to 8 columns so every Q view is TMA-aligned
        width = ((r_cap + 7) // 8) * 8
        if q_arena.shape[-1] != width:
            wide = torch.zeros(q_arena.shape[:-1] + (width,), device=q_arena.device, dtype=q_arena.dtype)
            wide[..., :r_cap] = q_arena[..., :r_cap]
            q_arena = wide
        self._arenas[key] = {"M": mom_arena, "Q": q_arena, "order": list(order)}
        c = self._ada_config
        for p, slot in zip(params, order):
            self._param_config[p] = cfg
            st = self.state[p]
            m, n = p.shape
            mult = self.param_groups[0]["rank_multiple_of"]
            init_r = mult * math.ceil(c["init_rank_fraction"] * min(m, n) / mult)
            init_r = int(min(max(1, init_r), r_cap))
            st["momentum"] = mom_arena[slot]
            st["Q"] = q_arena[slot][:, :r_cap]
            self._q_full[id(p)] = q_arena[slot]
            if "r" not in st:
                st.update({"r": init_r, "r_cap": r_cap, "transpose": cfg.is_transposed, "erank_ema": None,
                           "aerr_ema": None, "ada_step": 0})

    # ------------------------------------------------------------------ hooks
    def _active_q(self, params, order, Qb):
        if not self._adaptive_rank:
            return Qb, None
        slots = Qb.size(0)
        ranks = [0] * slots
        for p, s in zip(params, order):
            ranks[s] = int(self.state[p]["r"])
        width = Qb.shape[-1]
        r_max = min(width, ((max(ranks) + 7) // 8) * 8)
        Qw = Qb[:, :, :r_max]
        mask = (torch.arange(r_max, device=Qb.device).unsqueeze(0)
                < device_list(ranks, torch.int64, Qb.device).unsqueeze(1)).to(Qb.dtype)
        Qw.mul_(mask.unsqueeze(1))
        return Qw, ranks

    def _orth(self, P: Tensor, group: dict, ranks) -> Tensor:
        if ranks is None:
            return super()._orth(P, group, ranks)
        out = torch.zeros_like(P)
        by_rank: Dict[int, List[int]] = {}
        for i, r in enumerate(ranks):
            if r > 0:
                by_rank.setdefault(int(r), []).append(i)
        for r, idx in by_rank.items():
            it = device_list(idx, torch.int64, P.device)
            sub = P.index_select(0, it)[:, :, :r].contiguous()
            out[it, :, :r] = orthogonalize(sub, float(group["oversample"]))
        return out

    # ------------------------------------------------------------------ checkpoint
    # In adaptive mode ``momentum`` and ``Q`` are plain local tensors (shards of
    # a sharded parameter's state). The checkpoint view wraps them as DTensors
    # of the parameter's mesh (momentum with the parameter's placements, Q with
    # Dion's Q placements), so DCP stores every shard and reshards on load;
    # loading re-packs them into a local arena on the next step, as for Dion.
    # erank_ema / aerr_ema are None until first set; a flattened DCP checkpoint
    # (the container's format) cannot hold None, so they are left out while
    # None and put back on load.
    def _checkpoint_view(self, p: Tensor, st: Dict[str, Any]) -> Dict[str, Any]:
        out = {n: v for n, v in st.items() if v is not None}
        cfg = self._param_config.get(p)
        if not (self._adaptive_rank and isinstance(p, DTensor) and "r_cap" in st) or (
                cfg is not None and cfg.inner_shard_mesh_dim is not None):
            return out  # (with an inner shard the local tensors stay as they are)
        mom, Q = st.get("momentum"), st.get("Q")
        if mom is not None and not isinstance(mom, DTensor):
            out["momentum"] = DTensor.from_local(mom.contiguous(), p.device_mesh, p.placements, run_check=False,
                                                 shape=p.shape, stride=p.stride())
        if Q is not None and not isinstance(Q, DTensor) and cfg is not None:
            if cfg.Q_sharded_placements is None:
                self._q_placements(p, cfg)
            rows = p.shape[0] if st["transpose"] else p.shape[1]
            out["Q"] = DTensor.from_local(Q.contiguous(), p.device_mesh, cfg.Q_sharded_placements, run_check=False,
                                          shape=torch.Size((rows, Q.shape[1])), stride=(Q.shape[1], 1))
        return out

    def state_dict(self):
        sd = super().state_dict()
        params = [p for g in self.param_groups for p in g["params"]]
        sd["state"] = {k: self._checkpoint_view(params[k], st) if isinstance(k, int) and k < len(params)
                       else {n: v for n, v in st.items() if v is not None} for k, st in sd["state"].items()}
        return sd

    def load_state_dict(self, state_dict) -> None:
        super().load_state_dict(state_dict)
        for st in self.state.values():
            if "r_cap" in st:
                st.setdefault("erank_ema", None)
                st.setdefault("aerr_ema", None)

    def _after_update(self, group, params, order, sumsq, ranks) -> None:
        if ranks is None:
            return
        c = self._ada_config
        slots = device_list([order[i] for i in range(len(params))], torch.int64, sumsq.device)
        rs = device_list([ranks[order[i]] for i in range(len(params))], torch.int32, sumsq.device)
        # entropy effective rank of the active column norms (one kernel), one
        # device->host copy per shape group for the host-side rank schedule
        eranks = ops.effective_rank(sumsq, slots, rs).cpu().tolist()
        for p, er in zip(params, eranks):
            st = self.state[p]
            r, r_cap = st["r"], st["r_cap"]
            if math.isnan(er):
                er = float(r)
            b = c["erank_ema_beta"]
            st["erank_ema"] = er if st["erank_ema"] is None else b * st["erank_ema"] + (1 - b) * er
            st["ada_step"] += 1
            if st["ada_step"] % c.get("adapt_step", 1) != 0:
                continue
            desired = int(round(c["rank_scale"] * st["erank_ema"]))
            desired = min(max(c["rank_min"], desired), r_cap)
            desired = _quantize_int(desired, c["rank_quantize"])
            desired = min(max(c["rank_min"], desired), r_cap)
            if desired > r:
                r_next = min(desired, r + c["rank_step_up"])
            elif desired < r:
                r_next = max(desired, r - c["rank_step_down"])
            else:
                r_next = r
            r_next = int(min(max(c["rank_min"], r_next), r_cap))
            if r_next > r:
                Q = self._q_full[id(p)]
                # keyed by (shape, adaptation step, column range): identical on every
                # rank and after a resume (CUDA: Philox + column-normalise kernels)
                ops.keyed_unit_columns_(Q[:, r:r_next], 0x41445632, Q.shape[0], Q.shape[1], st["ada_step"], r,
                                        r_next)
            st["r"] = r_next

    # ------------------------------------------------------------------ diagnostics
    def _dion_params(self):
        idx = 0
        for group in self.param_groups:
            if group.get("algorithm", "dion") != "dion":
                continue
            for p in group["params"]:
                if p.ndim != 2:
                    continue
                yield idx, p
                idx += 1

    def get_rank(self) -> dict:
        if not self._adaptive_rank:
            return {}
        out = {}
        for idx, p in self._dion_params():
            st = self.state[p]
            if "r" in st:
                m, n = p.shape
                out[f"p{idx}_{m}x{n}"] = st["r"]
        return out

    def get_effective_rank(self) -> dict:
        if not self._adaptive_rank:
            return {}
        out = {}
        for idx, p in self._dion_params():
            st = self.state[p]
            if st.get("erank_ema") is not None:
                m, n = p.shape
                out[f"p{idx}_{m}x{n}"] = st["erank_ema"]
        return out

    def get_aerr(self) -> dict:
        if not self._adaptive_rank:
            return {}
        return {f"param_{idx}": self.state[p]["aerr_ema"] for idx, p in self._dion_params()
                if self.state[p].get("aerr_ema") is not None}
