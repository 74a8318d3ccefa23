"""Fused model-side ops (RMSNorm, rotary embedding, SwiGLU, cross-entropy).

The CUDA versions are sm_100a kernels of the ``dion_b200._C`` extension,
wrapped in autograd Functions; ``enabled(x)`` says whether a tensor takes the
fused path (CUDA, bf16, extension present, not disabled through
``DION_B200_FUSED=0``)."""
from __future__ import annotations

import os
from typing import Tuple

import torch
import torch.nn.functional as F

from ._ext import ext, has_ext

_DISABLED = os.environ.get("DION_B200_FUSED", "1") == "0"
_ADDNORM_DISABLED = os.environ.get("DION_B200_FUSED_ADDNORM", "1") == "0"


def enabled(x: torch.Tensor) -> bool:
    return (not _DISABLED) and x.is_cuda and x.dtype == torch.bfloat16 and has_ext() and hasattr(ext(), "rms_norm_fwd")


# ---------------------------------------------------------------- RMSNorm
class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], device=x.device, dtype=torch.float32)
        ext().rms_norm_fwd(x2, w, y, rstd, float(eps))
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, gy):
        x2, w, rstd = ctx.saved_tensors
        gy2 = gy.reshape(-1, gy.shape[-1]).contiguous()
        gx = torch.empty_like(x2)
        gw = torch.empty(w.shape, device=w.device, dtype=torch.float32)
        ext().rms_norm_bwd(gy2, x2, w, rstd, gx, gw)
        return gx.view(ctx.shape), gw.to(w.dtype), None


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return _RMSNorm.apply(x, w, eps)


class _AddRMSNorm(torch.autograd.Function):
    """h = x + a and y = rms_norm(h) * w in one pass (the residual add of a
    transformer block fused into the next norm); the backward adds the
    residual gradient into the norm's input gradient in the same pass."""

    @staticmethod
    def forward(ctx, x, a, w, eps):
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        a2 = a.reshape(-1, a.shape[-1]).contiguous()
        h = torch.empty_like(x2)
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], device=x.device, dtype=torch.float32)
        ext().add_rms_norm_fwd(x2, a2, w, h, y, rstd, float(eps))
        ctx.save_for_backward(h, w, rstd)
        ctx.shape = x.shape
        return h.view(x.shape), y.view(x.shape)

    @staticmethod
    def backward(ctx, gh, gy):
        h, w, rstd = ctx.saved_tensors
        gy2 = gy.reshape(-1, gy.shape[-1]).contiguous()
        gh2 = gh.reshape(-1, gh.shape[-1]).contiguous()
        gx = torch.empty_like(h)
        gw = torch.empty(w.shape, device=w.device, dtype=torch.float32)
        ext().rms_norm_bwd_res(gy2, h, w, rstd, gh2, gx, gw)
        g = gx.view(ctx.shape)
        return g, g, gw.to(w.dtype), None


def add_rms_enabled(x: torch.Tensor) -> bool:
    """Fused add + RMSNorm: bf16 rows of 1024-8192 (multiple of 256) features."""
    d = x.shape[-1]
    return (not _ADDNORM_DISABLED and enabled(x) and hasattr(ext(), "add_rms_norm_fwd") and d % 256 == 0
            and 1024 <= d <= 8192)


def add_rms_norm(x: torch.Tensor, a: torch.Tensor, w: torch.Tensor, eps: float):
    """Returns (x + a, rms_norm(x + a) * w)."""
    return _AddRMSNorm.apply(x, a, w, eps)


# ---------------------------------------------------------------- RoPE
class _Rope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, rope):
        qo = torch.empty_like(q, memory_format=torch.contiguous_format)
        ko = torch.empty_like(k, memory_format=torch.contiguous_format)
        ext().rope_fwd(q.contiguous(), k.contiguous(), rope, qo, ko, False)
        ctx.save_for_backward(rope)
        return qo, ko

    @staticmethod
    def backward(ctx, gq, gk):
        (rope,) = ctx.saved_tensors
        gqo = torch.empty_like(gq, memory_format=torch.contiguous_format)
        gko = torch.empty_like(gk, memory_format=torch.contiguous_format)
        ext().rope_fwd(gq.contiguous(), gk.contiguous(), rope, gqo, gko, True)
        return gqo, gko, None


def rope(q: torch.Tensor, k: torch.Tensor, table: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    return _Rope.apply(q, k, table)


# ---------------------------------------------------------------- SwiGLU
class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        a, b = a.contiguous(), b.contiguous()
        out = torch.empty_like(a)
        ext().swiglu_fwd(a, b, out)
        ctx.save_for_backward(a, b)
        return out

    @staticmethod
    def backward(ctx, go):
        a, b = ctx.saved_tensors
        ga = torch.empty_like(a)
        gb = torch.empty_like(b)
        ext().swiglu_bwd(go.contiguous(), a, b, ga, gb)
        return ga, gb


def swiglu(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return _SwiGLU.apply(a, b)


# ---------------------------------------------------------------- cross-entropy
def cross_entropy_fwd_bwd(logits: torch.Tensor, labels: torch.Tensor, grad_scale: float):
    """Return (sum of per-row losses (fp32 scalar), grad_scale * (softmax - onehot) in logits' dtype)."""
    if enabled(logits) and hasattr(ext(), "cross_entropy_fwd_bwd"):
        loss = torch.empty((), device=logits.device, dtype=torch.float32)
        grad = torch.empty_like(logits)
        ext().cross_entropy_fwd_bwd(logits.contiguous(), labels.contiguous(), grad, loss, float(grad_scale))
        return loss, grad
    lf = logits.float()
    lse = torch.logsumexp(lf, dim=-1)
    picked = lf.gather(1, labels.view(-1, 1)).squeeze(1)
    loss = (lse - picked).sum()
    p = torch.exp(lf - lse.unsqueeze(1))
    p.scatter_add_(1, labels.view(-1, 1), torch.full_like(picked.view(-1, 1), -1.0))
    return loss, (p * grad_scale).to(logits.dtype)
