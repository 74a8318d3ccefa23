"""AdaDion ("ANCHOR-MBP"): low-rank Dion with Cholesky QR, error feedback,
effective-rank adaptive rank with approximation-error quality control, and
an anchor blend of Q toward a periodically cached basis.

Behaviour of ada_dion/optim/adadion.py:60-441 (constructor defaults, state
keys M / Qbuf / r / tr / erank_ema / aerr_ema / Q_anchor / step, the
``_adadion_ws`` checkpoint stamp, getters). The momentum convention is
``B = M + G`` and ``M <- B - (1 - mu) * approx`` (no mu*M decay).

Legacy keyword aliases accepted: ``anchor_lambda`` -> ``anchor_alpha``,
``refresh_period`` -> ``anchor_period``, ``rank_fraction`` (a fraction of
min(m, n) used as the initial rank of each matrix).
"""
from __future__ import annotations

import math
from typing import Any, Dict, Optional

import torch
from torch.distributed.device_mesh import DeviceMesh

from ._lowrank import LowRankOptimizer, quantize_int

__all__ = ["AdaDion"]


class AdaDion(LowRankOptimizer):
    WS_KEY = "_adadion_ws"
    SEED_TAG = 0x4469_6F6E
    NULLABLE_STATE = ("erank_ema", "aerr_ema", "Q_anchor")
    DIAG_KEYS = ("r", "erank_ema", "aerr_ema")

    def __init__(
        self,
        params,
        lr: float = 0.02,
        mu: float = 0.95,
        init_rank: int = 64,
        adaptive_rank: bool = True,
        erank_ema_beta: float = 0.9,
        rho: float = 1.5,
        rank_min: int = 16,
        rank_max: int = 256,
        rank_quantize: int = 8,
        rank_warmup_steps: int = 10,
        warmup_rank: int = 128,
        rank_step_up: int = 16,
        rank_step_down: int = 8,
        use_quality_control: bool = True,
        aerr_ema_beta: float = 0.95,
        aerr_target: float = 0.08,
        aerr_up_margin: float = 0.15,
        aerr_down_margin: float = 0.15,
        use_anchor: bool = True,
        anchor_alpha: float = 0.1,
        anchor_period: int = 50,
        qbuf_max_cols: int = 256,
        weight_decay: float = 0.0,
        adamw_betas: tuple = (0.9, 0.95),
        adamw_eps: float = 1e-8,
        device_mesh: Optional[DeviceMesh] = None,
        **legacy,
    ):
        if "anchor_lambda" in legacy:
            anchor_alpha = float(legacy.pop("anchor_lambda"))
        if "refresh_period" in legacy:
            anchor_period = int(legacy.pop("refresh_period"))
        rank_fraction = legacy.pop("rank_fraction", None)
        for k in ("anchor_rho", "tau_lo", "tau_hi"):
            legacy.pop(k, None)
        if legacy:
            raise TypeError(f"AdaDion got unexpected keyword arguments {sorted(legacy)}")
        defaults = dict(
            lr=lr, mu=mu, init_rank=init_rank, adaptive_rank=adaptive_rank, erank_ema_beta=erank_ema_beta,
            rho=rho, rank_min=rank_min, rank_max=rank_max, rank_quantize=rank_quantize,
            rank_warmup_steps=rank_warmup_steps, warmup_rank=warmup_rank, rank_step_up=rank_step_up,
            rank_step_down=rank_step_down, use_quality_control=use_quality_control, aerr_ema_beta=aerr_ema_beta,
            aerr_target=aerr_target, aerr_up_margin=aerr_up_margin, aerr_down_margin=aerr_down_margin,
            use_anchor=use_anchor, anchor_alpha=anchor_alpha, anchor_period=anchor_period,
            qbuf_max_cols=qbuf_max_cols, weight_decay=weight_decay, adamw_betas=adamw_betas, adamw_eps=adamw_eps,
            rank_fraction=rank_fraction,
        )
        super().__init__(params, defaults, device_mesh)

    def _diag_name(self, i: int) -> str:
        return f"param_{i}"

    def _matrix_step(self, p, g: Dict[str, Any], st: Dict[str, Any]) -> None:
        eng = self.engine
        pl, mf, n, ml, ss, rc = self._geometry(p, g)
        if rc <= 0:
            return
        grad = self._local(p.grad)
        adaptive = g["adaptive_rank"]
        if len(st) == 0:
            init_rank = g["init_rank"]
            if g.get("rank_fraction") is not None:
                init_rank = max(1, int(math.ceil(g["rank_fraction"] * min(mf, n))))
            gi = dict(g, init_rank=init_rank)
            self._init_common(p, gi, st, g["qbuf_max_cols"] if adaptive else init_rank)
            st["erank_ema"] = None
            st["aerr_ema"] = None
            st["Q_anchor"] = None
        st["step"] += 1
        M, Qbuf, tr = st["M"], st["Qbuf"], st["tr"]
        re = int(max(1, min(g["rank_min"], rc, Qbuf.shape[1])))
        r = int(min(max(re, st["r"] if adaptive else g["init_rank"]), Qbuf.shape[1], rc))
        B = M + grad
        anchor = st["Q_anchor"] if g["use_anchor"] else None
        D, approx, Qn, R = eng.power_step(B, Qbuf, r, tr, ml, n, anchor, g["anchor_alpha"])
        self._write_q(st, Qn, r)
        D, _ = self._nan_guard(D)
        M.copy_(B - (1.0 - g["mu"]) * approx)
        lr, wd = g["lr"], g["weight_decay"]
        if wd:
            pl.mul_(1 - lr * wd)
        pl.add_(D, alpha=-(lr * ss))
        if g["use_anchor"] and (st["step"] % g["anchor_period"] == 0 or st["Q_anchor"] is None):
            st["Q_anchor"] = Qbuf.clone()
        if adaptive:
            self._adapt_rank(g, st, B, approx, R, r, re, rc, tr)

    def _adapt_rank(self, g, st, B, approx, R, r, re, rc, tr) -> None:
        eng = self.engine
        Qbuf = st["Qbuf"]
        cap = Qbuf.shape[1]
        if st["step"] <= g["rank_warmup_steps"]:
            des = max(re, int(min(g["warmup_rank"], rc, cap)))
            if des > r:
                self._refill(Qbuf, r, des, st["step"])
            st["r"] = des
            return
        sig = torch.linalg.vector_norm(R.float(), dim=0)
        if tr:
            sq = sig.pow(2)
            eng.all_reduce(sq)
            sig = sq.sqrt()
        sig = sig + 1e-12
        pr = sig / (sig.sum() + 1e-12)
        er = torch.exp(-(pr * torch.log(pr + 1e-12)).sum()).item()
        b = g["erank_ema_beta"]
        st["erank_ema"] = er if st["erank_ema"] is None else b * st["erank_ema"] + (1 - b) * er
        des = int(round(g["rho"] * st["erank_ema"]))
        if g["use_quality_control"]:
            ae = eng.rel_residual(B, approx)
            ab = g["aerr_ema_beta"]
            st["aerr_ema"] = ae if st["aerr_ema"] is None else ab * st["aerr_ema"] + (1 - ab) * ae
            if ae > max(g["aerr_target"], st["aerr_ema"] * (1 + g["aerr_up_margin"])):
                des = max(des, r + g["rank_step_up"])
            if ae < min(0.5 * g["aerr_target"], st["aerr_ema"] * (1 - g["aerr_down_margin"])):
                des = min(des, r - g["rank_step_down"])
        des = quantize_int(min(max(re, des), rc, cap), g["rank_quantize"])
        des = min(max(re, des), rc, cap)
        if des > r:
            rn = min(des, r + g["rank_step_up"])
        elif des < r:
            rn = max(des, r - g["rank_step_down"])
        else:
            rn = r
        rn = int(min(max(re, rn), rc, cap))
        if rn > r:
            self._refill(Qbuf, r, rn, st["step"])
        st["r"] = rn

    def get_effective_rank(self) -> Dict[str, float]:
        out = {}
        for i, p in self._matrix_params():
            if self._is_matrix(p):
                v = self.state[p].get("erank_ema")
                if v is not None:
                    out[f"param_{i}"] = v
        return out

    def get_aerr(self) -> Dict[str, float]:
        out = {}
        for i, p in self._matrix_params():
            if self._is_matrix(p):
                v = self.state[p].get("aerr_ema")
                if v is not None:
                    out[f"param_{i}"] = v
        return out

    def get_tail_ratio(self) -> Dict[str, float]:
        """Current ||(I - QQ^T) M|| / ||M|| per matrix (legacy diagnostic)."""
        out = {}
        for i, p in self._matrix_params():
            st = self.state[p]
            if self._is_matrix(p) and "M" in st:
                r = st["r"]
                Q = st["Qbuf"][:, :r]
                out[f"param_{i}"] = self.engine.tail(st["M"], Q, st["tr"])
        return out
