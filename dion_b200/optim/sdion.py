"""SDion (Skip-Dion): event-triggered power iterations.

Per step and matrix a mode is chosen from the subspace drift (vs. the last
refresh basis) and the tail energy of the momentum:
  skip      - reuse the cached basis (projection only), optional decaying
              anchor blend;
  consensus - full power step (the single-node form of the consensus step);
  recovery  - full power step, a second one when the tail is very large,
              then refresh the anchor;
  full      - plain Dion power step, refresh the anchor.
Behaviour of ada_dion/optim/sdion.py:62-421 (defaults, state keys, mode
rule, getters, ``_sdion_ws`` stamp). Momentum: M <- mu M + G, B = M + G.
"""
from __future__ import annotations

import math
from typing import Any, Dict, Optional

from torch.distributed.device_mesh import DeviceMesh

from ._lowrank import LowRankOptimizer, _mm, col_norm

__all__ = ["SDion"]


class SDion(LowRankOptimizer):
    WS_KEY = "_sdion_ws"
    SEED_TAG = 0x5344_696F
    NULLABLE_STATE = ("Q_anchor",)
    DIAG_KEYS = ("r", "_drift", "_tail", "_mode", "steps_skipped", "total_skips", "total_full", "total_consensus",
                 "total_recovery")

    def __init__(
        self,
        params,
        lr: float = 0.02,
        mu: float = 0.95,
        init_rank: int = 64,
        rank_min: int = 16,
        rank_max: int = 256,
        enable_skip: bool = True,
        tau_drift_safe: float = 0.5,
        tau_drift_consensus: float = 1.5,
        tau_tail_recovery: float = 0.4,
        max_skip: int = 10,
        enable_consensus: bool = True,
        sketch_dim: int = 0,
        consensus_lambda: float = 0.3,
        enable_anchor: bool = True,
        anchor_alpha0: float = 0.15,
        anchor_halflife: float = 20.0,
        enable_recovery: bool = True,
        qbuf_max_cols: int = 256,
        weight_decay: float = 0.0,
        adamw_betas: tuple = (0.9, 0.95),
        adamw_eps: float = 1e-8,
        device_mesh: Optional[DeviceMesh] = None,
    ):
        defaults = dict(
            lr=lr, mu=mu, init_rank=init_rank, rank_min=rank_min, rank_max=rank_max, enable_skip=enable_skip,
            tau_drift_safe=tau_drift_safe, tau_drift_consensus=tau_drift_consensus,
            tau_tail_recovery=tau_tail_recovery, max_skip=max_skip, enable_consensus=enable_consensus,
            sketch_dim=sketch_dim, consensus_lambda=consensus_lambda, enable_anchor=enable_anchor,
            anchor_alpha0=anchor_alpha0, anchor_halflife=anchor_halflife, enable_recovery=enable_recovery,
            qbuf_max_cols=qbuf_max_cols, weight_decay=weight_decay, adamw_betas=adamw_betas, adamw_eps=adamw_eps,
        )
        super().__init__(params, defaults, device_mesh)

    def _choose_mode(self, g, drift: float, tail: float, since: int) -> str:
        if not g["enable_skip"] or since <= 0:
            return "full"
        if drift < g["tau_drift_safe"] and tail < g["tau_tail_recovery"] and since < g["max_skip"]:
            return "skip"
        if g["enable_consensus"] and drift < g["tau_drift_consensus"] and tail < g["tau_tail_recovery"]:
            return "consensus"
        if g["enable_recovery"] and (tail > g["tau_tail_recovery"] or drift > g["tau_drift_consensus"]):
            return "recovery"
        return "full"

    def _matrix_step(self, p, g: Dict[str, Any], st: Dict[str, Any]) -> None:
        eng = self.engine
        pl, mf, n, ml, ss, rc = self._geometry(p, g)
        if rc <= 0:
            return
        grad = self._local(p.grad)
        if len(st) == 0:
            self._init_common(p, g, st, g["qbuf_max_cols"])
            st.update({"Q_anchor": None, "last_refresh": 0, "steps_skipped": 0, "total_skips": 0, "total_full": 0,
                       "total_consensus": 0, "total_recovery": 0})
        st["step"] += 1
        M, Qbuf, r, tr = st["M"], st["Qbuf"], st["r"], st["tr"]
        M.mul_(g["mu"]).add_(grad)
        B = M + grad
        d0 = ml if tr else n
        drift = eng.drift(Qbuf[:d0, :r], st["Q_anchor"], r, tr)
        tail = eng.tail(M, Qbuf[:d0, :r], tr)
        since = st["step"] - st["last_refresh"]
        mode = self._choose_mode(g, drift, tail, since)
        if mode == "skip":
            D, approx = eng.cheap_step(B, Qbuf, r, tr, ml, n)
            st["steps_skipped"] += 1
            st["total_skips"] += 1
            if g["enable_anchor"] and st["Q_anchor"] is not None:
                decay = g["anchor_alpha0"] * math.exp(-since / g["anchor_halflife"])
                if decay > 0.01:
                    ar = min(r, st["Q_anchor"].shape[1])
                    Qc = Qbuf[:d0, :r].clone()
                    Qc[:, :ar] = (1 - decay) * Qc[:, :ar] + decay * st["Q_anchor"][:d0, :ar]
                    Qc = col_norm(Qc) if not tr else eng.col_norm_dist(Qc)
                    D = _mm(_mm(B, Qc), Qc.T.contiguous()) if not tr else _mm(Qc, _mm(Qc.T.contiguous(), B))
        else:
            D, approx, Qn, _ = eng.power_step(B, Qbuf, r, tr, ml, n)
            self._write_q(st, Qn, r)
            if mode == "recovery" and tail > g["tau_tail_recovery"] * 1.5:
                D, approx, Qn, _ = eng.power_step(B, Qbuf, r, tr, ml, n)
                self._write_q(st, Qn, r)
            st["steps_skipped"] = 0
            if mode == "consensus":
                st["total_consensus"] += 1
            else:
                st["Q_anchor"] = Qbuf.clone()
                st["last_refresh"] = st["step"]
                st["total_recovery" if mode == "recovery" else "total_full"] += 1
        D, _ = self._nan_guard(D)
        M.copy_(B - (1.0 - g["mu"]) * approx)
        lr, wd = g["lr"], g["weight_decay"]
        if wd:
            pl.mul_(1 - lr * wd)
        pl.add_(D, alpha=-(lr * ss))
        st["_drift"], st["_tail"], st["_mode"] = drift, tail, mode

    def get_mode_counts(self) -> Dict[str, float]:
        c = {"skip": 0, "full": 0, "consensus": 0, "recovery": 0}
        for _, p in self._matrix_params():
            if not self._is_matrix(p):
                continue
            st = self.state[p]
            c["skip"] += st.get("total_skips", 0)
            c["full"] += st.get("total_full", 0)
            c["consensus"] += st.get("total_consensus", 0)
            c["recovery"] += st.get("total_recovery", 0)
        total = sum(c.values())
        return {**c, "total": total, "skip_rate": c["skip"] / max(total, 1)}
