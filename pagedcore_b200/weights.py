"""TinyLlama weight containers and the seeded random initialisation of config 3.

The field names are those of PagedCore's ``LayerWeights`` / ``TinyLlamaWeights``
(src/pagedcore/weights.py:54-73), so either package's weights work with
either decoder.  Checkpoint loading (weights.py:131-...) is out of this
package's scope: there is no network here, and BASELINE config 3 asks for
random-init weights.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

HIDDEN = 2048
INTERMEDIATE = 5632
VOCAB = 32000
LAYERS = 22
QUERY_HEADS = 32
KV_HEADS = 4
HEAD_DIM = 64


@dataclass(frozen=True, slots=True)
class LayerWeights:
    input_norm: Tensor           # [2048]
    q_proj: Tensor               # [2048, 2048]
    k_proj: Tensor               # [256, 2048]
    v_proj: Tensor               # [256, 2048]
    o_proj: Tensor               # [2048, 2048]
    post_attention_norm: Tensor  # [2048]
    gate_proj: Tensor            # [5632, 2048]
    up_proj: Tensor              # [5632, 2048]
    down_proj: Tensor            # [2048, 5632]


@dataclass(frozen=True, slots=True)
class TinyLlamaWeights:
    embedding: Tensor            # [32000, 2048]
    layers: tuple[LayerWeights, ...]
    final_norm: Tensor           # [2048]
    lm_head: Tensor              # [32000, 2048], untied from the embedding


def random_weights(
    seed: int,
    device: str | torch.device = "cpu",
    *,
    std: float = 0.02,
    layers: int = LAYERS,
    vocab: int = VOCAB,
    intermediate: int = INTERMEDIATE,
    generator_device: str | torch.device = "cpu",
) -> TinyLlamaWeights:
    """FP16 weights ~N(0, std), norm weights 1.0.

    Every matrix is drawn in a fixed order (embedding, then per layer q, k,
    v, o, gate, up, down, then the LM head).  Drawn on the CPU (the default)
    the same seed gives the same bits on any machine and device, which the
    golden fixtures rely on; ``generator_device`` = the GPU draws them there,
    seconds faster, for throughput runs whose values do not matter.
    """
    generator = torch.Generator(device=generator_device).manual_seed(seed)

    def matrix(rows: int, cols: int) -> Tensor:
        values = torch.randn(rows, cols, generator=generator, dtype=torch.float32, device=generator_device) * std
        return values.to(torch.float16).to(device)

    def norm() -> Tensor:
        return torch.ones(HIDDEN, dtype=torch.float16, device=device)

    embedding = matrix(vocab, HIDDEN)
    stack = []
    for _ in range(layers):
        q = matrix(QUERY_HEADS * HEAD_DIM, HIDDEN)
        k = matrix(KV_HEADS * HEAD_DIM, HIDDEN)
        v = matrix(KV_HEADS * HEAD_DIM, HIDDEN)
        o = matrix(HIDDEN, QUERY_HEADS * HEAD_DIM)
        gate = matrix(intermediate, HIDDEN)
        up = matrix(intermediate, HIDDEN)
        down = matrix(HIDDEN, intermediate)
        stack.append(LayerWeights(norm(), q, k, v, o, norm(), gate, up, down))
    lm_head = matrix(vocab, HIDDEN)
    return TinyLlamaWeights(embedding, tuple(stack), norm(), lm_head)
