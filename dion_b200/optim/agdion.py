"""AGDion (Anchor-Gap Dion): plain Dion geometry plus
  * H2 anchor: Q pulled toward the basis cached at the last refresh;
  * H3 gap: an extra power step when the momentum's tail energy outside the
    rank-r subspace is high;
  * event-triggered refresh of the anchor on drift / tail thresholds
    (bounded by min/max periods).
Behaviour of ada_dion/optim/agdion.py:59-371 (defaults, state keys,
``_agdion_ws`` stamp, getters). Momentum: M <- mu M + G, B = M + G.
"""
from __future__ import annotations

from typing import Any, Dict, Optional

from torch.distributed.device_mesh import DeviceMesh

from ._lowrank import LowRankOptimizer, _mm, col_norm

__all__ = ["AGDion"]


class AGDion(LowRankOptimizer):
    WS_KEY = "_agdion_ws"
    SEED_TAG = 0x4147_4469
    NULLABLE_STATE = ("Q_anchor",)
    DIAG_KEYS = ("r", "_drift", "_tail", "_did_extra", "_did_refresh", "_steps_since_refresh")

    def __init__(
        self,
        params,
        lr: float = 0.02,
        mu: float = 0.95,
        init_rank: int = 64,
        rank_min: int = 16,
        rank_max: int = 256,
        use_anchor: bool = True,
        anchor_alpha: float = 0.1,
        use_gap: bool = True,
        tau_tail_extra: float = 0.3,
        use_event_refresh: bool = True,
        tau_drift: float = 2.0,
        tau_tail_refresh: float = 0.4,
        max_period: int = 200,
        min_period: int = 10,
        qbuf_max_cols: int = 256,
        weight_decay: float = 0.0,
        adamw_betas: tuple = (0.9, 0.95),
        adamw_eps: float = 1e-8,
        device_mesh: Optional[DeviceMesh] = None,
    ):
        defaults = dict(
            lr=lr, mu=mu, init_rank=init_rank, rank_min=rank_min, rank_max=rank_max, use_anchor=use_anchor,
            anchor_alpha=anchor_alpha, use_gap=use_gap, tau_tail_extra=tau_tail_extra,
            use_event_refresh=use_event_refresh, tau_drift=tau_drift, tau_tail_refresh=tau_tail_refresh,
            max_period=max_period, min_period=min_period, qbuf_max_cols=qbuf_max_cols, weight_decay=weight_decay,
            adamw_betas=adamw_betas, adamw_eps=adamw_eps,
        )
        super().__init__(params, defaults, device_mesh)

    def _matrix_step(self, p, g: Dict[str, Any], st: Dict[str, Any]) -> None:
        eng = self.engine
        pl, mf, n, ml, ss, rc = self._geometry(p, g)
        if rc <= 0:
            return
        grad = self._local(p.grad)
        if len(st) == 0:
            self._init_common(p, g, st, g["qbuf_max_cols"])
            st.update({"Q_anchor": None, "last_refresh": 0})
        st["step"] += 1
        M, Qbuf, r, tr = st["M"], st["Qbuf"], st["r"], st["tr"]
        M.mul_(g["mu"]).add_(grad)
        B = M + grad
        D, approx, Qn, _ = eng.power_step(B, Qbuf, r, tr, ml, n)
        tail = eng.tail(M, Qn, tr)
        extra = False
        if g["use_gap"] and tail > g["tau_tail_extra"]:
            self._write_q(st, Qn, r)
            D, approx, Qn, _ = eng.power_step(B, Qbuf, r, tr, ml, n)
            extra = True
        drift = 0.0
        if g["use_anchor"] and st["Q_anchor"] is not None and g["anchor_alpha"] > 0:
            Qa = st["Q_anchor"]
            drift = eng.drift(Qn, Qa, r, tr)
            a = g["anchor_alpha"]
            ar = min(r, Qa.shape[1])
            Qn[:, :ar] = (1 - a) * Qn[:, :ar] + a * Qa[: Qn.shape[0], :ar]
            Qn = col_norm(Qn) if not tr else eng.col_norm_dist(Qn)
            if not tr:
                # non-transposed: the update becomes the projection on the blended basis
                D = _mm(_mm(B, Qn), Qn.T.contiguous())
        D, _ = self._nan_guard(D)
        self._write_q(st, Qn, r)
        M.copy_(B - (1.0 - g["mu"]) * approx)
        lr, wd = g["lr"], g["weight_decay"]
        if wd:
            pl.mul_(1 - lr * wd)
        pl.add_(D, alpha=-(lr * ss))
        since = st["step"] - st["last_refresh"]
        refresh = False
        if g["use_event_refresh"] and since >= g["min_period"]:
            refresh = drift > g["tau_drift"] or tail > g["tau_tail_refresh"]
        if since >= g["max_period"]:
            refresh = True
        if refresh or st["Q_anchor"] is None:
            st["Q_anchor"] = Qbuf.clone()
            st["last_refresh"] = st["step"]
        st.update({"_drift": drift, "_tail": tail, "_did_extra": extra, "_did_refresh": refresh,
                   "_steps_since_refresh": since})

    def get_drift(self) -> Dict[str, float]:
        return {f"p{i}": self.state[p]["_drift"] for i, p in self._matrix_params()
                if self._is_matrix(p) and "_drift" in self.state[p]}

    def get_tail(self) -> Dict[str, float]:
        return {f"p{i}": self.state[p]["_tail"] for i, p in self._matrix_params()
                if self._is_matrix(p) and "_tail" in self.state[p]}
