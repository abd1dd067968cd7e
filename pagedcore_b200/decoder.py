"""Paged prefill and one-token decode of TinyLlama over this package's KV path.

Drop-in for the paged half of PagedCore's decoder.py:

* ``prefill_paged`` (decoder.py:113-135): a dense causal forward of the
  prompt, then one ``KVAllocator.append`` of every layer's rotated K and V
  once the forward has succeeded.
* ``decode_paged`` (decoder.py:156-199): the reference's per-row schedule
  and semantics - single-request shapes for every GEMM, the new token's K/V
  written before the read so it is attended, the whole batch staged by one
  ``append_decode`` so a failure anywhere leaves every row unchanged.  The
  attention and the KV writes are this package's CUDA kernels; the module
  names the reference's tests patch (``paged_attention``, ``project_qkv``,
  ``final_logits``, ``F``, ...) are looked up from this module's globals.
  Since every row is computed alone, a row's logits do not depend on the
  rest of the batch, bit for bit.

``BatchedDecoder`` is the throughput form: per layer one Q/K/V GEMM and one
gate/up GEMM over the whole batch, the fused decode-layer launch (Q/K RoPE,
new-token KV write and attention in one kernel), and fused residual-add +
RMSNorm and SwiGLU-product kernels in place of their eager op chains.  Its
GEMMs see the batch and its norms sum in another order, so its rows may
differ from ``decode_paged`` in the last bits.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch
import torch.nn.functional as F
from torch import Tensor

from pagedcore_b200 import kernels
from pagedcore_b200.attention import paged_attention
from pagedcore_b200.dense import (
    apply_rope,
    dense_attention,
    final_logits,
    output_projection,
    project_qkv,
    rms_norm,
    swiglu,
)
from pagedcore_b200.engine_types import RequestId
from pagedcore_b200.kv_cache import KVAllocator
from pagedcore_b200.weights import HEAD_DIM, HIDDEN, KV_HEADS, LAYERS, QUERY_HEADS, TinyLlamaWeights

_CONTEXT_LIMIT = 2048


def _check_prompt(input_ids: Tensor, weights: TinyLlamaWeights) -> None:
    if input_ids.dtype != torch.int64 or input_ids.ndim != 2 or input_ids.shape[0] != 1:
        raise ValueError("input_ids must be int64 [1, tokens]")
    if input_ids.device != weights.embedding.device:
        raise ValueError("input_ids and weights must be on the same device")
    if not 1 <= input_ids.shape[1] <= _CONTEXT_LIMIT:
        raise ValueError("forward requires 1 to 2048 total cached token positions")


@torch.inference_mode()
def prefill(input_ids: Tensor, weights: TinyLlamaWeights) -> tuple[Tensor, list[tuple[Tensor, Tensor]]]:
    """Dense causal forward of one prompt: logits [1, T, V] and per layer (rotated K, V) [1, 4, T, 64]."""
    _check_prompt(input_ids, weights)
    tokens = input_ids.shape[1]
    positions = torch.arange(tokens, device=input_ids.device)[None]
    allowed = (positions[0, None, :] <= positions[0, :, None])[None, None]
    hidden = F.embedding(input_ids, weights.embedding)
    cache = []
    for layer in weights.layers:
        query, key, value = project_qkv(rms_norm(hidden, layer.input_norm), layer)
        query, key = apply_rope(query, key, positions)
        cache.append((key, value))
        hidden = hidden + output_projection(dense_attention(query, key, value, allowed), layer)
        hidden = hidden + swiglu(rms_norm(hidden, layer.post_attention_norm), layer)
    return final_logits(hidden, weights), cache


@torch.inference_mode()
def prefill_paged(
    input_ids: Tensor, weights: TinyLlamaWeights, allocator: KVAllocator, request_id: RequestId
) -> Tensor:
    """Prefill one admitted, empty request; return all prompt logits [1, T, V].

    The prompt's K/V reach the pool in one append after the forward, so a
    failed forward publishes nothing; reservation and cleanup stay with the
    caller.
    """
    if allocator.cached_length(request_id) != 0:
        raise ValueError("paged prefill requires an empty request cache")
    if len(weights.layers) != LAYERS:
        raise ValueError("paged prefill requires 22 decoder layers")
    logits, cache = prefill(input_ids, weights)
    # [1, 4, T, 64] per layer -> [22, T, 4, 64]
    keys = torch.stack([key[0].transpose(0, 1) for key, _ in cache])
    values = torch.stack([value[0].transpose(0, 1) for _, value in cache])
    allocator.append(request_id, keys, values)
    return logits


@torch.inference_mode()
def prefill_paged_fused(
    input_ids: Tensor, weights: TinyLlamaWeights, allocator: KVAllocator, request_id: RequestId
) -> Tensor:
    """Prefill a prompt chunk through the pool; return its logits [1, T, V].

    Unlike ``prefill_paged`` nothing dense is kept: per layer the chunk's K
    (rotated in the write) and V go straight to their pool slots, and the
    causal attention reads them back through the block table with the
    prefill attention kernel (token t of the chunk attends to positions
    0 .. start + t).  The request may already hold a cache (the chunk
    continues it).  Attention accumulates in FP32 as paged decode does, so logits match
    the dense FP16 prefill within tolerance, not bit for bit.  Positions are
    published only after the whole forward succeeds.
    """
    _check_prompt(input_ids, weights)
    if len(weights.layers) != LAYERS:
        raise ValueError("paged prefill requires 22 decoder layers")
    tokens = input_ids.shape[1]
    with allocator.prefill_append(request_id, tokens) as chunk:
        hidden = F.embedding(input_ids, weights.embedding)  # [1, T, 2048]
        for index, layer in enumerate(weights.layers):
            x = rms_norm(hidden, layer.input_norm)
            query = F.linear(x, layer.q_proj).view(tokens, QUERY_HEADS, HEAD_DIM)
            key = F.linear(x, layer.k_proj).view(tokens, KV_HEADS, HEAD_DIM)
            value = F.linear(x, layer.v_proj).view(tokens, KV_HEADS, HEAD_DIM)
            rotated = chunk.write_layer(index, key, value, query)
            attention = chunk.attend(index, rotated)
            hidden = hidden + F.linear(attention.view(1, tokens, HIDDEN), layer.o_proj)
            hidden = hidden + swiglu(rms_norm(hidden, layer.post_attention_norm), layer)
        logits = final_logits(hidden, weights)
    return logits


def _check_decode(input_ids: Tensor, weights: TinyLlamaWeights, request_ids: Sequence[RequestId]) -> None:
    if input_ids.dtype != torch.int64 or input_ids.ndim != 2 or input_ids.shape != (len(request_ids), 1):
        raise ValueError("input_ids must be int64 [batch, 1] matching request IDs")
    if input_ids.device != weights.embedding.device:
        raise ValueError("input_ids and weights must be on the same device")
    if len(weights.layers) != LAYERS:
        raise ValueError("paged decode requires 22 decoder layers")


def _decode_row(hidden: Tensor, position: Tensor, layer, index: int, allocator: KVAllocator,
                request: RequestId) -> Tensor:
    """One decoder layer for one row [1, 1, 2048] at its position [1, 1]."""
    query, key, value = project_qkv(rms_norm(hidden, layer.input_norm), layer)
    query, key = apply_rope(query, key, position)
    allocator.write_decode_layer(request, index, key[0, :, 0], value[0, :, 0])
    attention = paged_attention(query, allocator, request, layer_index=index, eager_rounding=False)
    hidden = hidden + output_projection(attention, layer)
    return hidden + swiglu(rms_norm(hidden, layer.post_attention_norm), layer)


@torch.inference_mode()
def decode_paged(
    input_ids: Tensor, weights: TinyLlamaWeights, allocator: KVAllocator, request_ids: tuple[RequestId, ...]
) -> Tensor:
    """One token for every request; returns logits [B, 1, V] in request order."""
    _check_decode(input_ids, weights, request_ids)
    lengths = [allocator.cached_length(request) for request in request_ids]
    positions = torch.tensor(lengths, dtype=torch.int64, device=input_ids.device)[:, None]
    with allocator.append_decode(request_ids):
        hidden = F.embedding(input_ids, weights.embedding)  # [B, 1, 2048]
        for index, layer in enumerate(weights.layers):
            rows = [
                _decode_row(hidden[row : row + 1], positions[row : row + 1], layer, index, allocator, request)
                for row, request in enumerate(request_ids)
            ]
            hidden = torch.cat(rows)
        return torch.cat([final_logits(hidden[row : row + 1], weights) for row in range(len(request_ids))])


class BatchedDecoder:
    """Batched one-token decode steps over a fixed set of weights.

    The Q/K/V and gate/up weights are concatenated once here, so each layer
    runs two batched GEMMs where the per-row path runs five per row.
    """

    def __init__(self, weights: TinyLlamaWeights) -> None:
        if len(weights.layers) != LAYERS:
            raise ValueError("paged decode requires 22 decoder layers")
        self.weights = weights
        self.qkv = [torch.cat((layer.q_proj, layer.k_proj, layer.v_proj)) for layer in weights.layers]
        self.gate_up = [torch.cat((layer.gate_proj, layer.up_proj)) for layer in weights.layers]
        if weights.embedding.is_cuda:
            kernels.linear_error_flag(weights.embedding.device)  # before any graph capture

    def forward(self, input_ids: Tensor, attend: Callable[[int, Tensor, Tensor, Tensor], Tensor]) -> Tensor:
        """The decoder stack for token ids [B, 1]; ``attend(layer, q, k, v)`` is the decode layer.

        q [B, 32, 64], k and v [B, 4, 64] are unrotated views of the layer's
        fused Q/K/V projection (rows 2560 elements apart); ``attend`` returns
        the FP16 attention [B, 32, 64].  Shared by ``step`` and the CUDA-graph
        form (``graph.DecoderStepGraph``), so both run the same op sequence.
        The residual stream is one FP16 [B, 2048] buffer; each RMSNorm takes
        the residual add before it in the same kernel (``kernels.add_rms_norm``)
        and SwiGLU's product is one kernel (``kernels.silu_mul``), with the
        rounding points of the reference's eager ops (dense.py:17-21, 84-91).
        Projections run ``kernels.linear``: this library's matrix-vector kernel
        for a single row, its tcgen05 split-K kernel up to
        ``kernels.TC_MAX_ROWS`` rows, the library GEMM above.  The output, gate/up and down
        projections hand their split sums straight to the next fused kernel,
        which adds them where it would have read the FP16 product.
        """
        weights = self.weights
        batch = input_ids.shape[0]
        q_width, kv_width = QUERY_HEADS * HEAD_DIM, KV_HEADS * HEAD_DIM
        hidden = F.embedding(input_ids, weights.embedding).view(batch, HIDDEN)  # updated in place
        x = torch.empty_like(hidden)
        delta = None  # the output still to be added to the residual stream
        linear = kernels.linear
        for index, layer in enumerate(weights.layers):
            kernels.add_rms_norm(hidden, delta, layer.input_norm, x)
            qkv = linear(x, self.qkv[index])
            query = qkv[:, :q_width].view(batch, QUERY_HEADS, HEAD_DIM)
            key = qkv[:, q_width : q_width + kv_width].view(batch, KV_HEADS, HEAD_DIM)
            value = qkv[:, q_width + kv_width :].view(batch, KV_HEADS, HEAD_DIM)
            # RoPE(Q, K) + new-token KV write + attention: one fused launch.
            attention = attend(index, query, key, value)
            delta = linear(attention.view(batch, HIDDEN), layer.o_proj, split_sums=True)
            kernels.add_rms_norm(hidden, delta, layer.post_attention_norm, x)
            gate_up = linear(x, self.gate_up[index], split_sums=True)
            delta = linear(kernels.silu_mul(gate_up), layer.down_proj, split_sums=True)
        kernels.add_rms_norm(hidden, delta, weights.final_norm, x)
        return linear(x, weights.lm_head).view(batch, 1, -1)

    @torch.inference_mode()
    def step(self, input_ids: Tensor, allocator: KVAllocator, request_ids: tuple[RequestId, ...]) -> Tensor:
        """One token for every request; returns logits [B, 1, V] in request order."""
        _check_decode(input_ids, self.weights, request_ids)
        with allocator.append_decode(request_ids):
            return self.forward(input_ids, allocator.decode_layer)

    @torch.inference_mode()
    def prefill(self, input_ids: Tensor, allocator: KVAllocator, request_id: RequestId) -> Tensor:
        """Prefill a prompt chunk [1, T] through the pool; return its logits [1, T, V].

        ``prefill_paged_fused`` on the batched step's ops: the T prompt tokens
        are the rows of ``forward`` (fused Q/K/V and gate/up GEMMs, fused
        residual add + RMSNorm and SwiGLU product), and each layer's attention
        writes the chunk's K (rotated) and V to its pool slots and runs the
        causal prefill kernel over the block table.  The request may already
        hold a cache (the chunk continues it); positions are published only
        after the whole forward succeeds.
        """
        _check_prompt(input_ids, self.weights)
        tokens = input_ids.shape[1]
        with allocator.prefill_append(request_id, tokens) as chunk:

            def attend(index: int, query: Tensor, key: Tensor, value: Tensor) -> Tensor:
                # Q is rotated in place inside the fused projection's output.
                return chunk.attend(index, chunk.write_layer(index, key, value, query, in_place=True))

            logits = self.forward(input_ids.view(tokens, 1), attend)
        return logits.view(1, tokens, -1)


def decode_batched(
    input_ids: Tensor, weights: TinyLlamaWeights, allocator: KVAllocator, request_ids: tuple[RequestId, ...]
) -> Tensor:
    """``decode_paged``'s signature on the batched path (builds a ``BatchedDecoder`` per call)."""
    return BatchedDecoder(weights).step(input_ids, allocator, request_ids)
