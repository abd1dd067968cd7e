"""TinyLlama dense math around the paged KV path (FP16 tensors, torch ops).

RMSNorm, the Q/K/V and output projections, RoPE, causal dense attention for
prompt prefill, SwiGLU and the LM head.  Each function performs the same
floating-point operations in the same order as PagedCore's dense.py, so on
one device the results match the reference bit for bit: the paged decoder's
tests compare logits and cached K with zero tolerance.  The GEMMs are plain
library GEMMs (torch.nn.functional.linear).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from pagedcore_b200 import rope
from pagedcore_b200.weights import HEAD_DIM, KV_HEADS, QUERY_HEADS, LayerWeights, TinyLlamaWeights

_GROUP = QUERY_HEADS // KV_HEADS


def rms_norm(hidden: Tensor, weight: Tensor) -> Tensor:
    """x * rsqrt(mean(x^2) + 1e-5) in FP32, rounded to FP16, times the FP16 scale (dense.py:17-21)."""
    x = hidden.float()
    scaled = x * torch.rsqrt(x.square().mean(dim=-1, keepdim=True) + 1e-5)
    return weight * scaled.to(hidden.dtype)


def project_qkv(hidden: Tensor, layer: LayerWeights) -> tuple[Tensor, Tensor, Tensor]:
    """[B, T, 2048] -> Q [B, 32, T, 64], K and V [B, 4, T, 64], unrotated (dense.py:24-30)."""
    batch, tokens, _ = hidden.shape
    heads = ((layer.q_proj, QUERY_HEADS), (layer.k_proj, KV_HEADS), (layer.v_proj, KV_HEADS))
    return tuple(F.linear(hidden, w).view(batch, tokens, n, HEAD_DIM).transpose(1, 2) for w, n in heads)


def rope_factors(positions: Tensor, dtype: torch.dtype) -> tuple[Tensor, Tensor]:
    """cos and sin [B, 1, T, 64] at int64 positions [B or 1, T].

    From the FP16 table that the reference's apply_rope builds (FP32 angles,
    one rounding; dense.py:48-54), the first half of each row repeated.
    """
    table = rope.device_table(positions.device)  # FP16 [2, 2048, 32]
    cos = table[0][positions].repeat(1, 1, 2).unsqueeze(1)
    sin = table[1][positions].repeat(1, 1, 2).unsqueeze(1)
    return cos.to(dtype), sin.to(dtype)


def rotate(tensor: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """x*cos + rot(x)*sin with rot(x) = (-x[32:], x[:32]), each product rounded (dense.py:56-59)."""
    half = tensor.shape[-1] // 2
    turned = torch.cat((-tensor[..., half:], tensor[..., :half]), dim=-1)
    return tensor * cos + turned * sin


def apply_rope(query: Tensor, key: Tensor, positions: Tensor) -> tuple[Tensor, Tensor]:
    """Rotate Q and K [B, heads, T, 64] at absolute positions [B or 1, T] (dense.py:33-61)."""
    if (
        positions.dtype != torch.int64
        or positions.ndim != 2
        or positions.shape[0] not in (1, query.shape[0])
        or positions.shape[1] != query.shape[2]
    ):
        raise ValueError("position_ids must be int64 [batch or 1, query tokens]")
    cos, sin = rope_factors(positions, query.dtype)
    return rotate(query, cos, sin), rotate(key, cos, sin)


def dense_attention(query: Tensor, key: Tensor, value: Tensor, allowed: Tensor) -> Tensor:
    """Causal GQA attention over dense K/V for prompt prefill (dense.py:69-81).

    FP16 scores scaled by 1/8, masked to the FP16 minimum where ``allowed`` is
    False, softmax in FP32 rounded to FP16, then P.V.
    """
    if allowed.dtype != torch.bool:
        raise ValueError("causal_mask must be boolean with True for allowed keys")
    keys = key.repeat_interleave(_GROUP, dim=1)
    values = value.repeat_interleave(_GROUP, dim=1)
    scores = torch.matmul(query, keys.transpose(-2, -1)) * (HEAD_DIM**-0.5)
    scores = scores.masked_fill(~allowed, torch.finfo(query.dtype).min)
    weights = F.softmax(scores, dim=-1, dtype=torch.float32).to(query.dtype)
    return torch.matmul(weights, values)


def dense_attention_fp32(query: Tensor, key: Tensor, value: Tensor, allowed: Tensor) -> Tensor:
    """The FP32 contiguous attention the reference uses to check paged decode (dense.py:91-99)."""
    keys = key.repeat_interleave(_GROUP, dim=1).float()
    values = value.repeat_interleave(_GROUP, dim=1).float()
    scores = torch.matmul(query.float(), keys.transpose(-2, -1)) * (HEAD_DIM**-0.5)
    scores = scores.masked_fill(~allowed, -torch.inf)
    return torch.matmul(scores.softmax(dim=-1), values).to(query.dtype)


def output_projection(attention: Tensor, layer: LayerWeights) -> Tensor:
    """[B, 32, T, 64] merged in head order -> [B, T, 2048] @ o_proj^T (dense.py:84-88)."""
    batch, _, tokens, _ = attention.shape
    return F.linear(attention.transpose(1, 2).reshape(batch, tokens, QUERY_HEADS * HEAD_DIM), layer.o_proj)


def swiglu(hidden: Tensor, layer: LayerWeights) -> Tensor:
    """down(silu(gate(x)) * up(x)) (dense.py:102-104)."""
    gated = F.silu(F.linear(hidden, layer.gate_proj))
    return F.linear(gated * F.linear(hidden, layer.up_proj), layer.down_proj)


def final_logits(hidden: Tensor, weights: TinyLlamaWeights) -> Tensor:
    """Final RMSNorm and the untied LM head (dense.py:107-109)."""
    return F.linear(rms_norm(hidden, weights.final_norm), weights.lm_head)
