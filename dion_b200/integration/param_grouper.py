"""Split a model's parameters into matrix / embedding / output / norm groups.

Same classification rules as ada_dion/integration/param_grouper.py:30-113
(torchtitan, GPT-2 and HF Llama naming), so every optimizer sees an
identical grouping: embeddings and the LM head are never orthonormalised,
2-D transformer projections are.
"""
from __future__ import annotations

from typing import Dict, List, NamedTuple

import torch.nn as nn

__all__ = ["ParamGroups", "group_params_for_hybrid", "count_params"]

_EMBED_TOKENS = ("tok_embeddings", "wte", "wpe", "embed_tokens", "embedding")
_HEAD_TOKENS = ("output", "lm_head", "head")
_MATRIX_PATTERNS = (
    "attention.wq", "attention.wk", "attention.wv", "attention.wo",
    "feed_forward.w1", "feed_forward.w2", "feed_forward.w3",
    "attn.c_attn", "attn.c_proj", "mlp.c_fc", "mlp.c_proj",
    "self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
    "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj",
)


class ParamGroups(NamedTuple):
    matrix_params: List[nn.Parameter]
    embed_params: List[nn.Parameter]
    output_params: List[nn.Parameter]
    norm_params: List[nn.Parameter]


def _kind(name: str, ndim: int) -> str:
    n = name.lower()
    if any(t in n for t in _EMBED_TOKENS):
        return "embed"
    if any(t in n.split(".") for t in _HEAD_TOKENS):
        return "output"
    if ndim >= 2 and any(p in n for p in _MATRIX_PATTERNS):
        return "matrix"
    return "norm"


def group_params_for_hybrid(model: nn.Module) -> ParamGroups:
    out: Dict[str, List[nn.Parameter]] = {"matrix": [], "embed": [], "output": [], "norm": []}
    for name, p in model.named_parameters():
        if p.requires_grad:
            out[_kind(name, p.ndim)].append(p)
    return ParamGroups(out["matrix"], out["embed"], out["output"], out["norm"])


def count_params(groups: ParamGroups) -> Dict[str, int]:
    c = {
        "matrix": sum(p.numel() for p in groups.matrix_params),
        "embed": sum(p.numel() for p in groups.embed_params),
        "output": sum(p.numel() for p in groups.output_params),
        "norm": sum(p.numel() for p in groups.norm_params),
    }
    c["total"] = sum(c.values())
    return c
