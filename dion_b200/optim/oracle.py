"""Plain-PyTorch single-matrix reference steps (the numerical oracle).

Each function restates the reference math (ada_dion/optim/adadion_v2.py:
857-997 for Dion, DION/muon.py:581-703 for Muon) in float64 without any
batching, sharding or fused kernels; tests compare the package's optimizers
against them.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch
from torch import Tensor

__all__ = ["dion_step", "muon_step", "newton_schulz_ref", "adamw_step", "lion_step"]


def newton_schulz_ref(G: Tensor, coeffs: Sequence[Tuple[float, float, float]], eps: float = 1e-7) -> Tensor:
    X = G.double()
    tall = X.size(-2) > X.size(-1)
    if tall:
        X = X.mT
    X = X / (X.norm() + eps)
    for a, b, c in coeffs:
        A = X @ X.mT
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    return X.mT if tall else X


def muon_step(X: Tensor, G: Tensor, M: Tensor, lr: float, mu: float, wd: float, nesterov: bool,
              coeffs, adjust: str = "spectral_norm", eps: float = 1e-7) -> Tuple[Tensor, Tensor]:
    """Returns (X_new, M_new) in float64."""
    M = mu * M.double() + G.double()
    U = mu * M + G.double() if nesterov else M
    O = newton_schulz_ref(U, coeffs, eps)
    fan_out, fan_in = X.shape
    if adjust == "spectral_norm":
        alr = lr * math.sqrt(fan_out / fan_in)
    elif adjust == "rms_norm":
        alr = lr * 0.2 * math.sqrt(max(fan_out, fan_in))
    elif adjust == "keller_muon":
        alr = lr * math.sqrt(max(1.0, fan_out / fan_in))
    else:
        alr = lr
    Xn = (1 - lr * wd) * X.double() - alr * O
    return Xn, M


def dion_step(X: Tensor, G: Tensor, M: Tensor, Q: Tensor, lr: float, mu: float, wd: float,
              eps: float = 1e-8) -> Tuple[Tensor, Tensor, Tensor]:
    """One single-device Dion step with an exact QR orthogonalisation.

    Returns (X_new, M_new, Q_new) in float64. Q has shape (n, r), or (m, r)
    when m < n (transposed orientation)."""
    X, G, M, Q = X.double(), G.double(), M.double(), Q.double()
    m, n = X.shape
    t = m < n
    M = M + G
    Mt = M.mT if t else M
    P = Mt @ Q
    if (M == 0).all():
        P = torch.zeros_like(P)
        R = Q.clone()
    else:
        P, _ = torch.linalg.qr(P)
        R = Mt.mT @ P
    upd_m = P @ R.mT
    M = M - (1 - mu) * (upd_m.mT if t else upd_m)
    Qn = R / (R.norm(dim=0, keepdim=True) + eps)
    u = P @ Qn.mT
    X = (1 - lr * wd) * X - math.sqrt(m / n) * lr * (u.mT if t else u)
    return X, M, Qn


def adamw_step(X, G, M, V, lr, b1, b2, wd, eps, step):
    X, G, M, V = X.double(), G.double(), M.double(), V.double()
    M = M + (1 - b1) * (G - M)
    V = V + (1 - b2) * (G * G - V)
    denom = V.sqrt() / math.sqrt(1 - b2**step) + eps
    X = X * (1 - lr * wd) - (lr / (1 - b1**step)) * M / denom
    return X, M, V


def lion_step(X, G, M, lr, b1, b2, wd):
    X, G, M = X.double(), G.double(), M.double()
    U = torch.sign(M + (1 - b1) * (G - M))
    M = M + (1 - b2) * (G - M)
    X = X * (1 - lr * wd) - lr * U
    return X, M
