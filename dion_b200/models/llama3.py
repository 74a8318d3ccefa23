"""Llama-3 style decoder with torchtitan-compatible parameter names.

FQNs match torchtitan's Llama3 (tok_embeddings, layers.<i>.attention.{wq,wk,
wv,wo}, layers.<i>.attention_norm, layers.<i>.feed_forward.{w1,w2,w3},
layers.<i>.ffn_norm, norm, output) so the param grouper, checkpoints and the
hybrid optimizer container see the same names as with the reference's model
(ada_dion/integration/config_registry.py:60-154 builds its Llama3 specs the
same way).

Compute is bf16 on the tensor cores: cuBLAS for the plain projections,
torch SDPA (flash/cuDNN) for attention with native grouped-query heads, and
the package's fused kernels for RMSNorm, rotary embedding, SwiGLU and the
chunked cross-entropy when they are available on the device.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace
from typing import Dict, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import layers as L
from ..parallel.sp import sp_column_linears, sp_row_linear

__all__ = ["Llama3Config", "Transformer", "LLAMA3_CONFIGS", "llama3_config"]


@dataclass
class Llama3Config:
    dim: int = 4096
    n_layers: int = 32
    n_heads: int = 32
    n_kv_heads: Optional[int] = None
    vocab_size: int = 128256
    ffn_dim: Optional[int] = None
    multiple_of: int = 256
    ffn_dim_multiplier: Optional[float] = None
    norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    max_seq_len: int = 8192
    depth_init: bool = True

    def hidden_dim(self) -> int:
        if self.ffn_dim is not None:
            return self.ffn_dim
        h = int(2 * (4 * self.dim) / 3)
        if self.ffn_dim_multiplier is not None:
            h = int(self.ffn_dim_multiplier * h)
        return self.multiple_of * ((h + self.multiple_of - 1) // self.multiple_of)

    @property
    def kv_heads(self) -> int:
        return self.n_kv_heads or self.n_heads

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    def num_params(self, include_embedding: bool = True) -> int:
        d, h, kv, hd = self.dim, self.hidden_dim(), self.kv_heads, self.head_dim
        attn = d * d * 2 + 2 * d * kv * hd
        ffn = 3 * d * h
        per_layer = attn + ffn + 2 * d
        n = self.n_layers * per_layer + d + self.vocab_size * d  # + output
        if include_embedding:
            n += self.vocab_size * d
        return n

    def flops_per_token(self, seq_len: int) -> int:
        """Training FLOPs per token: 6 * non-embedding params + attention (12*l*h*q*t)."""
        nparams = self.num_params(include_embedding=False)
        return 6 * nparams + 12 * self.n_layers * self.n_heads * self.head_dim * seq_len


LLAMA3_CONFIGS: Dict[str, Llama3Config] = {
    # CPU parity / golden-curve model: 4 layers, d=256, 4 heads, SwiGLU 1024, vocab 4096
    "tiny": Llama3Config(dim=256, n_layers=4, n_heads=4, n_kv_heads=4, vocab_size=4096, ffn_dim=1024,
                         rope_theta=10000.0, max_seq_len=256),
    "debug": Llama3Config(dim=256, n_layers=6, n_heads=16, n_kv_heads=16, vocab_size=2048, ffn_dim=768,
                          rope_theta=500000.0, max_seq_len=2048),
    # reference paper model (ada_dion/integration/config_registry.py:60-89)
    "160M": Llama3Config(dim=768, n_layers=12, n_heads=12, n_kv_heads=4, vocab_size=128256, ffn_dim=2048,
                         rope_theta=500000.0, max_seq_len=8192),
    # reference 320M model: 18 layers, full multi-head attention (config_registry.py:109-140)
    "320M": Llama3Config(dim=768, n_layers=18, n_heads=12, n_kv_heads=12, vocab_size=128256, ffn_dim=2048,
                         rope_theta=500000.0, max_seq_len=8192),
    "1B": Llama3Config(dim=2048, n_layers=16, n_heads=32, n_kv_heads=8, vocab_size=128256, ffn_dim=8192,
                       rope_theta=500000.0, max_seq_len=8192),
    "8B": Llama3Config(dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, vocab_size=128256, ffn_dim=14336,
                       rope_theta=500000.0, max_seq_len=8192),
}


def llama3_config(name: str, **overrides) -> Llama3Config:
    return replace(LLAMA3_CONFIGS[name], **overrides)


class Attention(nn.Module):
    def __init__(self, cfg: Llama3Config):
        super().__init__()
        self.n_heads = cfg.n_heads
        self.n_kv_heads = cfg.kv_heads
        self.head_dim = cfg.head_dim
        self.wq = nn.Linear(cfg.dim, cfg.n_heads * self.head_dim, bias=False)
        self.wk = nn.Linear(cfg.dim, self.n_kv_heads * self.head_dim, bias=False)
        self.wv = nn.Linear(cfg.dim, self.n_kv_heads * self.head_dim, bias=False)
        self.wo = nn.Linear(cfg.n_heads * self.head_dim, cfg.dim, bias=False)
        self.sp = None  # sequence-parallel TP group (parallel/sp.py), set by apply_tp

    def forward(self, x: torch.Tensor, rope: torch.Tensor) -> torch.Tensor:
        if self.sp is not None:
            # x: this rank's [N / T, D] token shard; q/k/v cover all tokens, this rank's heads
            bs, seqlen = self.sp.batch_shape
            q, k, v = sp_column_linears(self.sp, x, [self.wq.weight, self.wk.weight, self.wv.weight])
            q = q.view(bs, seqlen, -1, self.head_dim)
            k = k.view(bs, seqlen, -1, self.head_dim)
            v = v.view(bs, seqlen, -1, self.head_dim)
            q, k = L.apply_rope(q, k, rope)
            o = L.causal_attention(q, k, v)
            return sp_row_linear(self.sp, o.reshape(bs * seqlen, -1), self.wo.weight)
        bs, seqlen, _ = x.shape
        # -1 heads: under tensor parallelism each rank holds n_heads / tp of them
        q = self.wq(x).view(bs, seqlen, -1, self.head_dim)
        k = self.wk(x).view(bs, seqlen, -1, self.head_dim)
        v = self.wv(x).view(bs, seqlen, -1, self.head_dim)
        q, k = L.apply_rope(q, k, rope)
        o = L.causal_attention(q, k, v)  # [bs, seq, heads, hd]
        return self.wo(o.reshape(bs, seqlen, -1))


class FeedForward(nn.Module):
    def __init__(self, dim: int, hidden: int):
        super().__init__()
        self.w1 = nn.Linear(dim, hidden, bias=False)
        self.w2 = nn.Linear(hidden, dim, bias=False)
        self.w3 = nn.Linear(dim, hidden, bias=False)
        self.sp = None  # sequence-parallel TP group (parallel/sp.py), set by apply_tp

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.sp is not None:
            a, b = sp_column_linears(self.sp, x, [self.w1.weight, self.w3.weight])
            return sp_row_linear(self.sp, L.swiglu(a, b), self.w2.weight)
        return self.w2(L.swiglu(self.w1(x), self.w3(x)))


# ops whose outputs selective activation checkpointing keeps (everything else
# -- norms, rotary, SwiGLU, residual adds -- is recomputed in the backward)
_SAC_SAVE = None


def _sac_context():
    global _SAC_SAVE
    from torch.utils.checkpoint import CheckpointPolicy, create_selective_checkpoint_contexts

    if _SAC_SAVE is None:
        aten = torch.ops.aten
        names = ("mm", "addmm", "bmm", "_scaled_dot_product_flash_attention", "_scaled_dot_product_cudnn_attention",
                 "_scaled_dot_product_efficient_attention")
        _SAC_SAVE = {getattr(aten, n).default for n in names if hasattr(aten, n)}

    def policy(ctx, op, *args, **kwargs):
        return CheckpointPolicy.MUST_SAVE if op in _SAC_SAVE else CheckpointPolicy.PREFER_RECOMPUTE

    return create_selective_checkpoint_contexts(policy)


class TransformerBlock(nn.Module):
    def __init__(self, layer_id: int, cfg: Llama3Config):
        super().__init__()
        self.layer_id = layer_id
        self.ac_mode = "none"  # "none" | "full" | "op" (see Transformer.set_activation_checkpointing)
        self.attention = Attention(cfg)
        self.feed_forward = FeedForward(cfg.dim, cfg.hidden_dim())
        self.attention_norm = L.RMSNorm(cfg.dim, cfg.norm_eps)
        self.ffn_norm = L.RMSNorm(cfg.dim, cfg.norm_eps)
        self.weight_init_std = 0.02 / (2 * (layer_id + 1)) ** 0.5 if cfg.depth_init else 0.02 / (2 * cfg.n_layers) ** 0.5

    def _block(self, x: torch.Tensor, rope: torch.Tensor) -> torch.Tensor:
        h, n = self.ffn_norm.add_forward(x, self.attention(self.attention_norm(x), rope))
        return h + self.feed_forward(n)

    def forward(self, x: torch.Tensor, rope: torch.Tensor) -> torch.Tensor:
        if self.ac_mode == "none" or not torch.is_grad_enabled():
            return self._block(x, rope)
        from torch.utils.checkpoint import checkpoint

        if self.ac_mode == "op":
            return checkpoint(self._block, x, rope, use_reentrant=False, context_fn=_sac_context)
        return checkpoint(self._block, x, rope, use_reentrant=False)


class Transformer(nn.Module):
    def __init__(self, cfg: Llama3Config):
        super().__init__()
        self.cfg = cfg
        self.tok_embeddings = nn.Embedding(cfg.vocab_size, cfg.dim)
        self.layers = nn.ModuleDict({str(i): TransformerBlock(i, cfg) for i in range(cfg.n_layers)})
        self.norm = L.RMSNorm(cfg.dim, cfg.norm_eps)
        self.sp = None  # sequence-parallel TP group (parallel/sp.py), set by apply_tp
        self.output = nn.Linear(cfg.dim, cfg.vocab_size, bias=False)
        self.register_buffer("rope_cache", L.rope_table(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta), persistent=False)

    def set_activation_checkpointing(self, mode: str = "none", option: str = "1") -> None:
        """Activation checkpointing per transformer block (torchtitan's
        ``activation_checkpoint.mode`` / ``selective_ac_option``):
        ``full``: every block keeps only its input and recomputes the rest;
        ``selective`` with option ``op``: every block keeps its GEMM and
        attention outputs and recomputes the elementwise work;
        ``selective`` with an integer N: every N-th block is fully checkpointed.
        Checkpointing runs inside each block's forward, so parameter names
        (and checkpoints / optimizer groups) do not change."""
        blocks = list(self.layers.values())
        for i, b in enumerate(blocks):
            if mode == "none":
                b.ac_mode = "none"
            elif mode == "full":
                b.ac_mode = "full"
            elif mode == "selective" and option == "op":
                b.ac_mode = "op"
            elif mode == "selective":
                every = int(option)
                b.ac_mode = "full" if every > 0 and i % every == 0 else "none"
            else:
                raise ValueError(f"unknown activation checkpointing mode {mode!r}")

    @torch.no_grad()
    def init_weights(self, mode: str = "normal", std: float = 0.02, generator: Optional[torch.Generator] = None):
        """``normal``: every weight ~ N(0, std) (norm weights = 1);
        ``torchtitan``: truncated normal with depth-scaled output projections."""
        for name, p in self.named_parameters():
            if name.endswith("norm.weight") or name == "norm.weight":
                p.fill_(1.0)
                continue
            if mode == "normal":
                p.normal_(0.0, std, generator=generator)
            elif mode == "torchtitan":
                if name == "tok_embeddings.weight":
                    nn.init.normal_(p, generator=generator)
                elif name == "output.weight":
                    s = self.cfg.dim ** -0.5
                    nn.init.trunc_normal_(p, std=s, a=-3 * s, b=3 * s, generator=generator)
                else:
                    layer = self.layers[name.split(".")[1]]
                    s = 0.02 if any(k in name for k in ("wq", "wk", "wv", "w1")) else layer.weight_init_std
                    nn.init.trunc_normal_(p, std=s, a=-2.0, b=2.0, generator=generator)
            else:
                raise ValueError(mode)
        self.rope_cache = L.rope_table(self.cfg.head_dim, self.cfg.max_seq_len, self.cfg.rope_theta).to(
            self.rope_cache.device
        )

    def forward(self, tokens: torch.Tensor, labels: Optional[torch.Tensor] = None,
                return_hidden: bool = False) -> torch.Tensor:
        """Logits, or with ``labels`` the mean next-token cross-entropy computed
        chunk-wise without materialising fp32 logits. (The loss lives in
        ``forward`` so FSDP's root hooks unshard the LM head for it.)"""
        seqlen = tokens.shape[1]
        sp = self.sp
        if sp is not None:
            # sequence parallelism: this rank embeds and carries its shard of the flattened tokens
            sp.batch_shape = (tokens.shape[0], seqlen)
            h = self.tok_embeddings(sp.shard_rows(tokens.reshape(-1)))
        else:
            h = self.tok_embeddings(tokens)
        rope = self.rope_cache[:seqlen].float()
        for layer in self.layers.values():
            h = layer(h, rope)
        h = self.norm(h)
        if labels is not None:
            if sp is not None:
                # this rank's share of the mean loss over all N tokens (the TP
                # ranks' shares sum to it; replicated-parameter gradients are
                # summed over TP after backward)
                return L.linear_cross_entropy(h, self.output.weight, sp.shard_rows(labels.reshape(-1))) / sp.T
            return L.linear_cross_entropy(h, self.output.weight, labels)
        if return_hidden:
            return h
        return self.output(h)

    def loss(self, tokens: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        return self(tokens, labels)
