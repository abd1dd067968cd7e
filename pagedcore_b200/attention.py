"""Block-table decode attention (drop-in for src/pagedcore/attention.py).

``paged_attention`` keeps the reference's single-request signature, checks and
errors (attention.py:14-30) and computes the same quantity - FP32 scores of
the FP16 query against FP16 K pages, one softmax over the valid context, FP32
weighted sum of V, one FP16 rounding - with the split-K sm_100a kernel.
``paged_decode_attention`` is the batched form used by the decode step.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
from torch import Tensor

from pagedcore_b200.engine_types import RequestId
from pagedcore_b200.kv_cache import KVAllocator


def _check_layer(layer_index: int) -> None:
    if type(layer_index) is not int or not 0 <= layer_index < 22:
        raise ValueError("layer_index must identify one of the 22 decoder layers")


@torch.inference_mode()
def paged_attention(
    query: Tensor,
    allocator: KVAllocator,
    request_id: RequestId,
    *,
    layer_index: int,
    eager_rounding: bool = False,
) -> Tensor:
    """Attend one FP16 query [1, 32, 1, 64] over one request's pages at a layer."""
    if query.shape != (1, 32, 1, 64) or query.dtype != torch.float16:
        raise ValueError("query must be FP16 [1, 32, 1, 64]")
    _check_layer(layer_index)
    batch = allocator.decode_batch((request_id,), layer_index=layer_index)
    if query.device != allocator.pool.device:
        raise ValueError("query and KV cache must be on the same device")
    if eager_rounding:
        raise NotImplementedError(
            "eager_rounding replays the reference's FP16 forensic paths, which are not part of the B200 KV path"
        )
    out = allocator.attend(batch, query.detach().reshape(1, 32, 64), layer_index=layer_index)
    return out.reshape(1, 32, 1, 64)


@torch.inference_mode()
def paged_decode_attention(
    query: Tensor,
    allocator: KVAllocator,
    request_ids: Sequence[RequestId],
    *,
    layer_index: int,
    out: Tensor | None = None,
) -> Tensor:
    """Attend FP16 queries [B, 32, 64] (row b for request_ids[b]) at one layer."""
    if query.ndim != 3 or query.shape[1:] != (32, 64) or query.dtype != torch.float16:
        raise ValueError("query must be FP16 [batch, 32, 64]")
    if query.shape[0] != len(request_ids):
        raise ValueError("query rows must match request_ids")
    _check_layer(layer_index)
    batch = allocator.decode_batch(request_ids, layer_index=layer_index)
    if query.device != allocator.pool.device:
        raise ValueError("query and KV cache must be on the same device")
    return allocator.attend(batch, query, layer_index=layer_index, out=out)
