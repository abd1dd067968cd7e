"""Oracle of block-table decode attention - test infrastructure only.

``paged_attention`` restates src/pagedcore/attention.py:32-53 in numpy:
FP32 scores page by page (q @ K_page^T, then * 64**-0.5), one FP32 softmax
over the valid context, FP32 P.V accumulated page by page, one FP16 rounding.
``dense_fp64`` is the independent FP64 reference of the reference's own tests
(tests/unit/test_attention.py:173-179).
"""

from __future__ import annotations

import numpy as np


def paged_attention(
    pool: np.ndarray, layer: int, query: np.ndarray, blocks: list[int] | tuple[int, ...], length: int
) -> np.ndarray:
    """query FP16 [32, 64]; pool FP16 [22, 2, N, 16, 4, 64] -> FP16 [32, 64]."""
    grouped = query.reshape(4, 8, 64).astype(np.float32)
    scores = np.empty((4, 8, length), dtype=np.float32)
    start = 0
    for logical, physical in enumerate(blocks):
        valid = min(16, length - logical * 16)
        key = pool[layer, 0, physical, :valid].astype(np.float32)  # [valid, 4, 64]
        scores[..., start : start + valid] = np.matmul(grouped, key.transpose(1, 2, 0)) * np.float32(0.125)
        start += valid
    shifted = np.exp(scores - scores.max(axis=-1, keepdims=True))
    probabilities = shifted / shifted.sum(axis=-1, keepdims=True)
    out = np.zeros((4, 8, 64), dtype=np.float32)
    start = 0
    for logical, physical in enumerate(blocks):
        valid = min(16, length - logical * 16)
        value = pool[layer, 1, physical, :valid].astype(np.float32)  # [valid, 4, 64]
        out += np.matmul(probabilities[..., start : start + valid], value.transpose(1, 0, 2))
        start += valid
    return out.reshape(32, 64).astype(np.float16)


def dense_fp64(query: np.ndarray, key: np.ndarray, value: np.ndarray) -> np.ndarray:
    """query [32, 64], key/value [L, 4, 64] -> FP16 [32, 64], in FP64."""
    heads = []
    for head in range(32):
        scores = query[head].astype(np.float64) @ key[:, head // 8].astype(np.float64).T / 8.0
        weights = np.exp(scores - scores.max())
        weights /= weights.sum()
        heads.append(weights @ value[:, head // 8].astype(np.float64))
    return np.stack(heads).astype(np.float16)


def gather_dense(pool: np.ndarray, layer: int, blocks, length: int) -> tuple[np.ndarray, np.ndarray]:
    """The valid K and V rows [L, 4, 64] of a request, in position order."""
    blocks = np.asarray(blocks, dtype=np.int64)
    key = pool[layer, 0, blocks].reshape(-1, 4, 64)[:length]
    value = pool[layer, 1, blocks].reshape(-1, 4, 64)[:length]
    return key, value
