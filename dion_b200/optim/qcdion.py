"""QCDion (Quality-Controlled Dion): plain Dion geometry, with
  * a quality gate g_t = clip(exp(-rho (z_t - EMA(z))), [1/gamma, gamma]) on
    the composite score z = w_q q + w_d d + w_e e (residual q, subspace drift
    d of Q Q^T, error-feedback burden e) scaling the step;
  * an extra power step when q_t > tau_extra;
  * a temporary rank doubling after boost_k consecutive bad steps, dropped
    back to the base rank once quality recovers.
Behaviour of ada_dion/optim/qcdion.py:60-353 (defaults, state keys,
diagnostics, ``_qcdion_ws`` stamp).
"""
from __future__ import annotations

import math
from typing import Any, Dict, Optional

import torch
from torch.distributed.device_mesh import DeviceMesh

from ._lowrank import LowRankOptimizer, _mm

__all__ = ["QCDion"]


class QCDion(LowRankOptimizer):
    WS_KEY = "_qcdion_ws"
    SEED_TAG = 0x5143_4469
    NULLABLE_STATE = ("Q_prev_proj",)
    DIAG_KEYS = ("r", "_q_t", "_d_t", "_e_t", "_z_t", "_g_t", "_D_fro", "z_ema", "_extra_step", "bad_streak")

    def __init__(
        self,
        params,
        lr: float = 0.02,
        mu: float = 0.95,
        init_rank: int = 64,
        rank_min: int = 16,
        rank_max: int = 256,
        use_quality_gate: bool = True,
        gate_rho: float = 0.3,
        gate_gamma: float = 1.15,
        gate_beta: float = 0.99,
        gate_w_q: float = 1.0,
        gate_w_d: float = 0.3,
        gate_w_e: float = 0.3,
        use_extra_power: bool = True,
        tau_extra: float = 0.2,
        use_rank_boost: bool = True,
        tau_rank: float = 0.25,
        boost_k: int = 5,
        qbuf_max_cols: int = 256,
        weight_decay: float = 0.0,
        adamw_betas: tuple = (0.9, 0.95),
        adamw_eps: float = 1e-8,
        device_mesh: Optional[DeviceMesh] = None,
    ):
        defaults = dict(
            lr=lr, mu=mu, init_rank=init_rank, rank_min=rank_min, rank_max=rank_max,
            use_quality_gate=use_quality_gate, gate_rho=gate_rho, gate_gamma=gate_gamma, gate_beta=gate_beta,
            gate_w_q=gate_w_q, gate_w_d=gate_w_d, gate_w_e=gate_w_e, use_extra_power=use_extra_power,
            tau_extra=tau_extra, use_rank_boost=use_rank_boost, tau_rank=tau_rank, boost_k=boost_k,
            qbuf_max_cols=qbuf_max_cols, weight_decay=weight_decay, adamw_betas=adamw_betas, adamw_eps=adamw_eps,
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
            st.update({"r_base": st["r"], "z_ema": 0.1, "bad_streak": 0, "Q_prev_proj": None})
        st["step"] += 1
        M, Qbuf, r, tr = st["M"], st["Qbuf"], st["r"], st["tr"]
        mu = g["mu"]
        M.mul_(mu).add_(grad)
        B = M + grad
        D, approx, Qn, _ = eng.power_step(B, Qbuf, r, tr, ml, n)
        proj = _mm(Qn, Qn.T.contiguous())
        has_prev = st["Q_prev_proj"] is not None and proj.shape == st["Q_prev_proj"].shape
        dproj = proj - st["Q_prev_proj"] if has_prev else torch.zeros((), device=proj.device)
        # the step's four measurements: one all-reduce, one host read (the
        # projector difference is replicated unless the basis is row-sharded)
        m_sq, q_sq, e_sq, d_sq = eng.sq_sums(M, B - approx, B - (1.0 - mu) * approx - M, dproj,
                                             reduce=[True, True, True, bool(tr)])
        M_fro = math.sqrt(m_sq) + 1e-12
        q_t = math.sqrt(q_sq) / (M_fro + 1e-12)
        d_t = math.sqrt(d_sq) if has_prev else 0.0
        st["Q_prev_proj"] = proj.clone()
        e_t = math.sqrt(e_sq) / (M_fro + 1e-12)
        z_t = g["gate_w_q"] * q_t + g["gate_w_d"] * d_t + g["gate_w_e"] * e_t
        extra = False
        if g["use_extra_power"] and q_t > g["tau_extra"]:
            self._write_q(st, Qn, r)
            D, approx, Qn, _ = eng.power_step(B, Qbuf, r, tr, ml, n)
            extra = True
        if g["use_quality_gate"]:
            st["z_ema"] = g["gate_beta"] * st["z_ema"] + (1 - g["gate_beta"]) * z_t
            g_t = max(1.0 / g["gate_gamma"], min(g["gate_gamma"], math.exp(-g["gate_rho"] * (z_t - st["z_ema"]))))
        else:
            g_t = 1.0
        D, bad = self._nan_guard(D)
        if bad:
            g_t = 0.0
        self._write_q(st, Qn, r)
        M.copy_(B - (1.0 - mu) * approx)
        lr, wd = g["lr"], g["weight_decay"]
        if wd:
            pl.mul_(1 - lr * wd)
        pl.add_(D, alpha=-(lr * ss * g_t))
        if g["use_rank_boost"]:
            if q_t > g["tau_rank"]:
                st["bad_streak"] += 1
                if st["bad_streak"] >= g["boost_k"]:
                    rn = min(r * 2, rc, Qbuf.shape[1])
                    if rn > r:
                        self._refill(Qbuf, r, rn, st["step"])
                    st["r"] = rn
                    st["bad_streak"] = 0
            else:
                st["bad_streak"] = 0
                if r > st["r_base"] and q_t < g["tau_rank"] * 0.5:
                    st["r"] = st["r_base"]
        st.update({"_q_t": q_t, "_d_t": d_t, "_e_t": e_t, "_z_t": z_t, "_g_t": g_t,
                   "_D_fro": D.float().norm().item(), "_extra_step": extra})
