"""Seeded synthetic workloads of the BASELINE configurations.

PagedCore publishes no benchmark inputs (it has no benchmark suite), so every
configuration is generated here from a seed, deterministically on any machine
(numpy PCG64 streams keyed by (seed, purpose, index)).  Values are FP16
~N(0, 1) unless stated.  Tests, golden-fixture generation and ``bench.py``
all draw their inputs from these functions.

- ``attention_case``   config 1: 4 rows, contexts {17, 100, 513, 2048}, pool
  512 blocks, block tables from a seeded permutation of the free list.
- ``churn_ops`` / ``append_case``  config 2: pool 4096 blocks, 10k-op
  allocate/release churn, then 8 prompts U[1, 2048] and 256 one-token appends.
- ``decode_case``      configs 4/5: ragged contexts, churned tables, a decode
  step's Q/K/V per layer.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

LAYERS = 22
KV_HEADS = 4
QUERY_HEADS = 32
HEAD_DIM = 64
BLOCK_TOKENS = 16


def rng(seed: int, *key: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, *key])))


def normal_f16(generator: np.random.Generator, shape: tuple[int, ...]) -> np.ndarray:
    return generator.standard_normal(shape, dtype=np.float32).astype(np.float16)


def blocks_for(tokens: int) -> int:
    return (tokens + BLOCK_TOKENS - 1) // BLOCK_TOKENS


# ---------------------------------------------------------------------------
# Config 1: single-layer batched decode attention.
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class AttentionCase:
    num_blocks: int
    lengths: tuple[int, ...]
    free_order: np.ndarray  # initial free stack (bottom..top), a permutation of the pool
    keys: tuple[np.ndarray, ...]  # per row FP16 [22, L, 4, 64] (already rotated; appended as-is)
    values: tuple[np.ndarray, ...]
    query: np.ndarray  # FP16 [rows, 32, 64] (FP32 N(0,1) rounded to FP16)


def attention_case(
    seed: int = 1, lengths: tuple[int, ...] = (17, 100, 513, 2048), num_blocks: int = 512, layers: int = LAYERS
) -> AttentionCase:
    free_order = rng(seed, 1, 0).permutation(num_blocks).astype(np.int32)
    keys = tuple(normal_f16(rng(seed, 1, 1, i), (layers, n, KV_HEADS, HEAD_DIM)) for i, n in enumerate(lengths))
    values = tuple(normal_f16(rng(seed, 1, 2, i), (layers, n, KV_HEADS, HEAD_DIM)) for i, n in enumerate(lengths))
    query = normal_f16(rng(seed, 1, 3), (len(lengths), QUERY_HEADS, HEAD_DIM))
    return AttentionCase(num_blocks, tuple(lengths), free_order, keys, values, query)


# ---------------------------------------------------------------------------
# Config 2: KV append / scatter after allocator churn.
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class ChurnOp:
    kind: str  # "create" (reserve + append `tokens`) or "release"
    request: int
    credits: int = 0
    tokens: int = 0


def churn_ops(
    seed: int, num_blocks: int, count: int = 10_000, target_live: int = 300, max_tokens: int = 128
) -> list[ChurnOp]:
    """A seeded alloc/free sequence; each create reserves room for +1 token.

    The op list depends only on the seed (the reserved-credit total is tracked
    here exactly as the allocator tracks it), so any allocator replaying it
    must end with the same tables.
    """
    generator = rng(seed, 2, 0)
    live: list[tuple[int, int]] = []
    reserved = 0
    next_request = 0
    ops: list[ChurnOp] = []
    for _ in range(count):
        release = bool(live) and generator.random() < len(live) / (2.0 * target_live)
        tokens = int(generator.integers(1, max_tokens + 1))
        credits = blocks_for(tokens + 1)
        if not release and reserved + credits > num_blocks // 2:
            release = bool(live)
        if release:
            index = int(generator.integers(len(live)))
            request, credit = live.pop(index)
            reserved -= credit
            ops.append(ChurnOp("release", request))
        else:
            ops.append(ChurnOp("create", next_request, credits, tokens))
            live.append((next_request, credits))
            reserved += credits
            next_request += 1
    return ops


def churn_fill(op_index: int, tokens: int) -> tuple[np.ndarray, np.ndarray]:
    """Cheap deterministic K/V [22, tokens, 4, 64] for churn appends (a tag per op)."""
    tag = np.float16((op_index % 2000) / 8.0)
    key = np.full((LAYERS, tokens, KV_HEADS, HEAD_DIM), tag, dtype=np.float16)
    return key, (-key - np.float16(1)).astype(np.float16)


@dataclass(frozen=True)
class PromptWrite:
    request: int
    credits: int
    key: np.ndarray  # FP16 [22, T, 4, 64], unrotated
    value: np.ndarray


@dataclass(frozen=True)
class DecodeWrite:
    requests: tuple[int, ...]  # staged order
    key: np.ndarray  # FP16 [22, B, 4, 64], unrotated
    value: np.ndarray


@dataclass(frozen=True)
class AppendCase:
    num_blocks: int
    churn: list[ChurnOp]
    prompts: list[PromptWrite]
    decode: DecodeWrite


def append_case(
    seed: int = 2,
    num_blocks: int = 4096,
    churn_count: int = 10_000,
    prompt_count: int = 8,
    decode_rows: int = 256,
    max_prompt: int = 2048,
    churn_tokens: int = 128,
) -> AppendCase:
    churn = churn_ops(seed, num_blocks, churn_count, max_tokens=churn_tokens)
    live = {}
    for op in churn:
        if op.kind == "create":
            live[op.request] = op.tokens
        else:
            del live[op.request]
    generator = rng(seed, 2, 1)
    first = 1_000_000
    prompts = []
    for i in range(prompt_count):
        tokens = int(generator.integers(1, max_prompt + 1))
        tokens = min(tokens, 2047)
        prompts.append(
            PromptWrite(
                first + i,
                blocks_for(tokens + 1),
                normal_f16(rng(seed, 2, 2, i), (LAYERS, tokens, KV_HEADS, HEAD_DIM)),
                normal_f16(rng(seed, 2, 3, i), (LAYERS, tokens, KV_HEADS, HEAD_DIM)),
            )
        )
    candidates = [p.request for p in prompts] + sorted(live)
    if len(candidates) < decode_rows:
        raise ValueError("churn left too few live requests for the decode rows")
    chosen = [p.request for p in prompts] + [
        int(r) for r in generator.choice(sorted(live), size=decode_rows - len(prompts), replace=False)
    ]
    order = generator.permutation(len(chosen))
    requests = tuple(chosen[i] for i in order)
    decode = DecodeWrite(
        requests,
        normal_f16(rng(seed, 2, 4), (LAYERS, len(requests), KV_HEADS, HEAD_DIM)),
        normal_f16(rng(seed, 2, 5), (LAYERS, len(requests), KV_HEADS, HEAD_DIM)),
    )
    return AppendCase(num_blocks, churn, prompts, decode)


# ---------------------------------------------------------------------------
# Configs 4/5: batched ragged decode.
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class DecodeCase:
    num_blocks: int
    lengths: np.ndarray  # int32 [B] cached lengths before the step
    credits: np.ndarray  # int32 [B]
    churn: list[ChurnOp]


def decode_lengths(seed: int, batch: int, low: int = 1, high: int = 2048 - 64) -> np.ndarray:
    return rng(seed, 4, 0).integers(low, high + 1, size=batch).astype(np.int32)


def decode_case(seed: int = 4, batch: int = 256, steps: int = 64, churn_count: int = 2_000) -> DecodeCase:
    """Contexts U[1, 2048-64] (room for ``steps`` more tokens), churned pool."""
    lengths = decode_lengths(seed, batch, high=2048 - steps)
    credits = np.array([blocks_for(int(n) + steps) for n in lengths], dtype=np.int32)
    need = int(credits.sum())
    num_blocks = need + need // 8 + 64
    churn = churn_ops(seed, num_blocks // 8, churn_count, target_live=32, max_tokens=64)
    return DecodeCase(num_blocks, lengths, credits, churn)


def decode_step_inputs(seed: int, batch: int, step: int, layers: int = LAYERS) -> tuple[np.ndarray, ...]:
    """Unrotated Q [L, B, 32, 64], K/V [L, B, 4, 64] of one decode step."""
    q = normal_f16(rng(seed, 5, step, 0), (layers, batch, QUERY_HEADS, HEAD_DIM))
    k = normal_f16(rng(seed, 5, step, 1), (layers, batch, KV_HEADS, HEAD_DIM))
    v = normal_f16(rng(seed, 5, step, 2), (layers, batch, KV_HEADS, HEAD_DIM))
    return q, k, v
