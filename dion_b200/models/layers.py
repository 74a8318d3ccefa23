"""Building blocks of the Llama model: RMSNorm, rotary embedding, causal
grouped-query attention, SwiGLU and a memory-lean linear + cross-entropy.

Each op uses the package's fused sm_100a kernel for CUDA bf16 inputs when
the extension provides it, and plain PyTorch otherwise (CPU runs and
autograd reference)."""
from __future__ import annotations

import math
from typing import Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..ops import fused as _fused

__all__ = [
    "RMSNorm",
    "rope_table",
    "apply_rope",
    "causal_attention",
    "swiglu",
    "linear_cross_entropy",
]


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _fused.enabled(x):
            return _fused.rms_norm(x, self.weight, self.eps)
        return F.rms_norm(x.float(), (x.shape[-1],), self.weight.float(), self.eps).to(x.dtype)

    def add_forward(self, x: torch.Tensor, a: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """(x + a, norm(x + a)): the residual add fused into the norm where the kernel applies."""
        if _fused.add_rms_enabled(x) and a.dtype == x.dtype and a.shape == x.shape:
            return _fused.add_rms_norm(x, a, self.weight, self.eps)
        h = x + a
        return h, self(h)

    def reset_parameters(self):
        nn.init.ones_(self.weight)


def rope_table(head_dim: int, max_seq_len: int, theta: float) -> torch.Tensor:
    """[max_seq_len, head_dim/2, 2] table of (cos, sin), fp32."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    t = torch.arange(max_seq_len, dtype=torch.float64)
    ang = torch.outer(t, inv)
    return torch.stack([ang.cos(), ang.sin()], dim=-1).float()


def apply_rope(q: torch.Tensor, k: torch.Tensor, rope: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Rotate interleaved (even, odd) pairs of the head dim; q,k: [b, s, h, d]."""
    if _fused.enabled(q):
        return _fused.rope(q, k, rope)
    return _rope_ref(q, rope), _rope_ref(k, rope)


def _rope_ref(x: torch.Tensor, rope: torch.Tensor) -> torch.Tensor:
    xf = x.float().reshape(*x.shape[:-1], -1, 2)
    c = rope[: x.shape[1], None, :, 0]
    s = rope[: x.shape[1], None, :, 1]
    x0, x1 = xf[..., 0], xf[..., 1]
    out = torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1)
    return out.flatten(-2).to(x.dtype)


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """q: [b, s, hq, d], k/v: [b, s, hkv, d] -> [b, s, hq, d]."""
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    gqa = qt.shape[1] != kt.shape[1]
    o = F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, enable_gqa=gqa)
    return o.transpose(1, 2)


def swiglu(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if _fused.enabled(a):
        return _fused.swiglu(a, b)
    return F.silu(a) * b


class _LinearCE(torch.autograd.Function):
    """loss = mean CE(h @ W^T, labels) with the gradient computed chunk by
    chunk during forward, so the [tokens, vocab] logits never exist in fp32
    all at once."""

    @staticmethod
    def forward(ctx, h, W, labels, chunk: int):
        T = h.shape[0]
        grad_h = torch.empty_like(h)
        grad_W = torch.zeros_like(W, dtype=torch.float32)
        total = torch.zeros((), device=h.device, dtype=torch.float32)
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            hc = h[s:e]
            logits = hc @ W.t()
            lab = labels[s:e]
            loss_c, g = _fused.cross_entropy_fwd_bwd(logits, lab, 1.0 / T)
            total += loss_c
            grad_h[s:e] = g @ W
            # grad_W (fp32) += g^T @ hc on the tensor cores, accumulating in place
            ops.matmul(g.t(), hc, out=grad_W, C=grad_W, beta=1.0)
        ctx.save_for_backward(grad_h, grad_W.to(W.dtype))
        return total / T

    @staticmethod
    def backward(ctx, go):
        grad_h, grad_W = ctx.saved_tensors
        return grad_h * go, grad_W * go, None, None


def linear_cross_entropy(h: torch.Tensor, W: torch.Tensor, labels: torch.Tensor, chunk: int = 8192) -> torch.Tensor:
    h2 = h.reshape(-1, h.shape[-1])
    lab = labels.reshape(-1)
    if not h.is_cuda:
        return F.cross_entropy((h2 @ W.t()).float(), lab)
    if not (torch.is_grad_enabled() and (h.requires_grad or W.requires_grad)):
        # evaluation: the same chunked loss without the gradient products
        T = h2.shape[0]
        total = torch.zeros((), device=h.device, dtype=torch.float32)
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            loss_c, _ = _fused.cross_entropy_fwd_bwd(h2[s:e] @ W.t(), lab[s:e], 1.0 / T)
            total += loss_c
        return total / T
    return _LinearCE.apply(h2, W, lab, chunk)
