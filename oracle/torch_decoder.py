"""Device-side comparators of the decoder - TEST INFRASTRUCTURE ONLY.

Torch restatements of the two comparators PagedCore itself uses to check
paged decode on a GPU, so the tests can run them on the same device as the
CUDA path (the numpy oracle cannot run the full TinyLlama model in seconds):

* ``ContiguousDecoder`` - the reference's contiguous-cache decoder:
  ``decoder.prefill`` (the dense FP16 prompt forward) then
  ``decoder.decode(..., fp32_attention=True)`` per token
  (src/pagedcore/decoder.py:103-110, 138-153, 202-240; the decode attention
  is dense.py:91-99: full FP32 matmuls and softmax over the whole history,
  one FP16 rounding of the attention output, no page traversal).  The
  reference's GPU parity test uses exactly this pair as its blocking
  comparator (tests/gpu/test_decoder_parity.py:205-240).
* ``paged_attention_fp32`` - the reference's own page loop
  (src/pagedcore/attention.py:32-53) in torch: FP32 scores page by page,
  one softmax, FP32 P.V page by page, one FP16 rounding.  Patched in place
  of the CUDA kernel it tells which part of a logit difference comes from
  the kernel's arithmetic and which from elsewhere.

The non-attention maths (RMSNorm, projections, RoPE, SwiGLU, LM head) are
``pagedcore_b200.dense``, which performs the reference's dense.py ops in the
reference's order: the reference's comparator shares those components with
the paged path too (docs/NUMERICAL_POLICY.md, "Integrated comparison").
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from pagedcore_b200.dense import (
    apply_rope,
    dense_attention,
    dense_attention_fp32,
    final_logits,
    output_projection,
    project_qkv,
    rms_norm,
    swiglu,
)


class ContiguousDecoder:
    """One request's greedy decode over a contiguous FP16 K/V history.

    ``prefill(ids [1, T])`` and ``decode(ids [1, 1])`` return logits
    [1, tokens, V]; K (rotated) and V of every position are kept per layer as
    [1, 4, positions, 64], as decoder.ContiguousCache holds them.
    """

    def __init__(self, weights) -> None:
        self.weights = weights
        self.layers: list[tuple[Tensor, Tensor]] | None = None

    @property
    def length(self) -> int:
        return 0 if self.layers is None else int(self.layers[0][0].shape[2])

    @torch.inference_mode()
    def _forward(self, input_ids: Tensor, fp32_attention: bool) -> Tensor:
        # decoder.py:202-240; prefill keeps the FP16 dense attention (dense.py:69-81).
        weights = self.weights
        offset, tokens = self.length, input_ids.shape[1]
        if offset + tokens > 2048:
            raise ValueError("forward requires 1 to 2048 total cached token positions")
        device = input_ids.device
        positions = torch.arange(offset, offset + tokens, device=device)[None]
        key_positions = torch.arange(offset + tokens, device=device)
        allowed = (key_positions[None, :] <= positions[0, :, None])[None, None]
        hidden = F.embedding(input_ids, weights.embedding)
        layers = []
        for index, layer in enumerate(weights.layers):
            query, key, value = project_qkv(rms_norm(hidden, layer.input_norm), layer)
            query, key = apply_rope(query, key, positions)
            if self.layers is not None:
                key = torch.cat((self.layers[index][0], key), dim=2)
                value = torch.cat((self.layers[index][1], value), dim=2)
            layers.append((key, value))
            attention = (dense_attention_fp32 if fp32_attention else dense_attention)(query, key, value, allowed)
            hidden = hidden + output_projection(attention, layer)
            hidden = hidden + swiglu(rms_norm(hidden, layer.post_attention_norm), layer)
        self.layers = layers
        return final_logits(hidden, weights)

    def prefill(self, input_ids: Tensor) -> Tensor:
        if self.layers is not None:
            raise ValueError("prefill needs an empty cache")
        return self._forward(input_ids, fp32_attention=False)

    def decode(self, input_ids: Tensor) -> Tensor:
        if input_ids.shape != (1, 1):
            raise ValueError("decode requires exactly one token with shape [1, 1]")
        return self._forward(input_ids, fp32_attention=True)


@torch.inference_mode()
def paged_attention_fp32(query: Tensor, allocator, request_id, *, layer_index: int,
                         eager_rounding: bool = False) -> Tensor:
    """attention.py:32-53 over the allocator's pages, in torch on the pool's device."""
    if eager_rounding:
        raise NotImplementedError("the forensic FP16 replays are not restated")
    grouped = query.reshape(4, 8, 64).float()
    scores = torch.empty((4, 8, 2048), dtype=torch.float32, device=query.device)
    length = 0
    for key, _ in allocator.iter_layer_blocks(request_id, layer_index=layer_index):
        stop = length + key.shape[0]
        scores[..., length:stop] = torch.matmul(grouped, key.permute(1, 2, 0).float()) * (64**-0.5)
        length = stop
    probabilities = scores[..., :length].softmax(dim=-1)
    output = torch.zeros_like(grouped)
    start = 0
    for _, value in allocator.iter_layer_blocks(request_id, layer_index=layer_index):
        stop = start + value.shape[0]
        output.add_(torch.matmul(probabilities[..., start:stop], value.transpose(0, 1).float()))
        start = stop
    return output.reshape(1, 32, 1, 64).half()
