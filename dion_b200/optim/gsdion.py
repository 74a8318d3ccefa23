"""GSDion (Guarded Scale-Dion): Dion's low-rank step with step-size
safeguards. The update P Q^T of rank r has Frobenius norm sqrt(r); GSDion
  1. divides it by sqrt(r) (rank normalisation);
  2. scales by a centred relative scalar s_t = clip(exp(-rho (log RMS(G) -
     EMA)), [1/gamma, gamma]);
  3. matches RMS(update) to RMS(M) and clips with a trust region
     alpha_t = min(1, tau / q_t) on the residual quality q_t;
  4. moves the rank with residual thresholds and hysteresis, refreshes Q
     periodically or on residual spikes;
  5. optionally pre-balances G by row/column RMS EMAs (MuonEq) and blends Q
     toward an anchor.
Behaviour of ada_dion/optim/gsdion.py:78-460 (defaults, state keys,
diagnostics, ``_gsdion_ws`` stamp).
"""
from __future__ import annotations

import math
from typing import Any, Dict, Optional

import torch
from torch.distributed.device_mesh import DeviceMesh

from ._lowrank import LowRankOptimizer, quantize_int

__all__ = ["GSDion"]


def _rms(X) -> torch.Tensor:
    return X.float().pow(2).mean().sqrt()


class GSDion(LowRankOptimizer):
    WS_KEY = "_gsdion_ws"
    SEED_TAG = 0x4753_4469
    NULLABLE_STATE = ("log_rms_ema", "Q_anchor")
    DIAG_KEYS = ("r", "_q_t", "_s_t", "_s_raw", "_c_t", "_alpha_t", "_m_t", "_dw_fro", "_dw_rms", "_grad_rms",
                 "_update_rms", "q_ema")

    def __init__(
        self,
        params,
        lr: float = 0.02,
        mu: float = 0.95,
        init_rank: int = 64,
        rank_min: int = 16,
        rank_max: int = 256,
        rank_quantize: int = 8,
        rank_normalize: bool = True,
        use_adaptive_scalar: bool = True,
        scalar_beta: float = 0.99,
        scalar_rho: float = 0.3,
        scalar_gamma: float = 1.2,
        use_rms_matching: bool = True,
        use_trust_region: bool = True,
        trust_tau: float = 1.0,
        use_residual_rank: bool = True,
        tau_up: float = 0.15,
        tau_down: float = 0.05,
        hysteresis_k: int = 5,
        rank_warmup_steps: int = 10,
        warmup_rank: int = 128,
        refresh_period: int = 100,
        refresh_spike: float = 0.5,
        use_pre_balance: bool = False,
        balance_beta: float = 0.99,
        use_anchor: bool = False,
        anchor_alpha: float = 0.1,
        anchor_period: int = 50,
        qbuf_max_cols: int = 256,
        weight_decay: float = 0.0,
        adamw_betas: tuple = (0.9, 0.95),
        adamw_eps: float = 1e-8,
        device_mesh: Optional[DeviceMesh] = None,
    ):
        defaults = dict(
            lr=lr, mu=mu, init_rank=init_rank, rank_min=rank_min, rank_max=rank_max, rank_quantize=rank_quantize,
            rank_normalize=rank_normalize, use_adaptive_scalar=use_adaptive_scalar, scalar_beta=scalar_beta,
            scalar_rho=scalar_rho, scalar_gamma=scalar_gamma, use_rms_matching=use_rms_matching,
            use_trust_region=use_trust_region, trust_tau=trust_tau, use_residual_rank=use_residual_rank,
            tau_up=tau_up, tau_down=tau_down, hysteresis_k=hysteresis_k, rank_warmup_steps=rank_warmup_steps,
            warmup_rank=warmup_rank, refresh_period=refresh_period, refresh_spike=refresh_spike,
            use_pre_balance=use_pre_balance, balance_beta=balance_beta, use_anchor=use_anchor,
            anchor_alpha=anchor_alpha, anchor_period=anchor_period, qbuf_max_cols=qbuf_max_cols,
            weight_decay=weight_decay, adamw_betas=adamw_betas, adamw_eps=adamw_eps,
        )
        super().__init__(params, defaults, device_mesh)

    def _rms_all(self, X, tr: bool) -> float:
        """RMS over the whole (possibly row-sharded) matrix."""
        if not tr:
            return _rms(X).item()
        # every row shard holds the same number of entries: one all-reduce of the sum of squares
        (s,) = self.engine.sq_sums(X)
        return math.sqrt(s / (X.numel() * self.engine.world_size()))

    def _matrix_step(self, p, g: Dict[str, Any], st: Dict[str, Any]) -> None:
        eng = self.engine
        pl, mf, n, ml, ss, rc = self._geometry(p, g)
        if rc <= 0:
            return
        grad = self._local(p.grad)
        if len(st) == 0:
            self._init_common(p, g, st, g["qbuf_max_cols"])
            st.update({"log_rms_ema": None, "q_ema": 0.1, "good_streak": 0, "Q_anchor": None})
            if g["use_pre_balance"]:
                st["Dr_ema"] = torch.ones(ml, device=pl.device, dtype=torch.float32)
                st["Dc_ema"] = torch.ones(n, device=pl.device, dtype=torch.float32)
        st["step"] += 1
        M, Qbuf, tr = st["M"], st["Qbuf"], st["tr"]
        dt = M.dtype
        cap = Qbuf.shape[1]
        re = int(max(1, min(g["rank_min"], rc, cap)))
        r = int(min(max(re, st["r"] if g["use_residual_rank"] else g["init_rank"]), cap, rc))

        if g["use_pre_balance"]:
            row_sq = grad.float().pow(2).sum(dim=1)
            col_sq = grad.float().pow(2).sum(dim=0)
            eng.all_reduce(col_sq)
            if tr:
                eng.all_reduce(row_sq)
            b = g["balance_beta"]
            st["Dr_ema"].mul_(b).add_(row_sq, alpha=1 - b)
            st["Dc_ema"].mul_(b).add_(col_sq, alpha=1 - b)
            gu = (grad.float() * st["Dr_ema"].clamp(min=1e-12).rsqrt().unsqueeze(1)
                  * st["Dc_ema"].clamp(min=1e-12).rsqrt().unsqueeze(0)).to(dt)
        else:
            gu = grad

        grad_rms = self._rms_all(grad, tr)
        if g["use_adaptive_scalar"]:
            lg = math.log(grad_rms + 1e-12)
            b = g["scalar_beta"]
            st["log_rms_ema"] = lg if st["log_rms_ema"] is None else b * st["log_rms_ema"] + (1 - b) * lg
            s_raw = math.exp(-g["scalar_rho"] * (lg - st["log_rms_ema"]))
            s_t = max(1.0 / g["scalar_gamma"], min(g["scalar_gamma"], s_raw))
        else:
            s_t = s_raw = 1.0

        M.mul_(g["mu"]).add_(gu)
        B = M + gu
        anchor = st["Q_anchor"] if g["use_anchor"] else None
        D_raw, approx, Qn, _ = eng.power_step(B, Qbuf, r, tr, ml, n, anchor, g["anchor_alpha"])
        self._write_q(st, Qn, r)
        D_raw, _ = self._nan_guard(D_raw)

        q_t = eng.rel_residual(B, approx)
        st["q_ema"] = 0.95 * st["q_ema"] + 0.05 * q_t
        D = D_raw / math.sqrt(r) if (g["rank_normalize"] and r > 0) else D_raw
        c_t = self._rms_all(M, tr) / (self._rms_all(D, tr) + 1e-12) if g["use_rms_matching"] else 1.0
        alpha_t = min(1.0, g["trust_tau"] / (q_t + 1e-12)) if g["use_trust_region"] else 1.0
        m_t = alpha_t * c_t * s_t
        lr, wd = g["lr"], g["weight_decay"]
        step_scale = lr * ss * m_t
        if not math.isfinite(step_scale):
            # a non-finite momentum (e.g. a NaN gradient) makes the RMS-matched
            # scale NaN even though the guard zeroed D: skip the update instead
            # of writing NaN into the weights
            step_scale = 0.0
        dw_fro = D.float().norm().item() * abs(step_scale)
        dw_rms = _rms(D).item() * abs(step_scale)

        M.copy_(B - (1.0 - g["mu"]) * approx)
        if wd:
            pl.mul_(1 - lr * wd)
        pl.add_(D, alpha=-step_scale)

        if g["use_anchor"] and (st["step"] % g["anchor_period"] == 0 or st["Q_anchor"] is None):
            st["Q_anchor"] = Qbuf.clone()
        warm = g["rank_warmup_steps"]
        if ((st["step"] % g["refresh_period"] == 0) or (q_t > g["refresh_spike"])) and st["step"] > warm:
            gen = torch.Generator(device=pl.device)
            gen.manual_seed(0x5246 + st["step"])
            self._refill(Qbuf, 0, r, st["step"], gen)
        if g["use_residual_rank"] and st["step"] > warm:
            if q_t > g["tau_up"]:
                st["good_streak"] = 0
                rn = min(r * 2, rc, cap)
            elif q_t < g["tau_down"]:
                st["good_streak"] += 1
                rn = max(r // 2, re) if st["good_streak"] >= g["hysteresis_k"] else r
                if st["good_streak"] >= g["hysteresis_k"]:
                    st["good_streak"] = 0
            else:
                st["good_streak"] = 0
                rn = r
            rn = quantize_int(min(max(re, rn), rc, cap), g["rank_quantize"])
            rn = int(min(max(re, rn), rc, cap))
            if rn > r:
                self._refill(Qbuf, r, rn, st["step"])
            st["r"] = rn
        elif st["step"] <= warm:
            des = max(re, int(min(g["warmup_rank"], rc, cap)))
            if des > r:
                self._refill(Qbuf, r, des, st["step"])
            st["r"] = des
        st.update({"_q_t": q_t, "_s_t": s_t, "_s_raw": s_raw, "_c_t": c_t, "_alpha_t": alpha_t, "_m_t": m_t,
                   "_dw_fro": dw_fro, "_dw_rms": dw_rms, "_grad_rms": grad_rms, "_update_rms": _rms(D).item()})
