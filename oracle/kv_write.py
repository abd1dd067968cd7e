"""Oracle of the KV writes into the pool - test infrastructure only.

The pool is a numpy FP16 array [22, 2, blocks, 16, 4, 64]
(src/pagedcore/kv_cache.py:39-43).  ``write_rows`` is the copy of
KVAllocator.append (kv_cache.py:161-172) and write_decode_layer
(kv_cache.py:244-245): row t of every layer goes to slot id slots[t] =
physical_block * 16 + slot.
"""

from __future__ import annotations

import numpy as np

from oracle import rope


def new_pool(num_blocks: int, fill: float = np.nan) -> np.ndarray:
    return np.full((22, 2, num_blocks, 16, 4, 64), fill, dtype=np.float16)


def write_rows(
    pool: np.ndarray, layer_begin: int, key: np.ndarray, value: np.ndarray, slots: np.ndarray
) -> None:
    """key/value FP16 [layers, T, 4, 64] -> pool[layer_begin + l, 0|1, slot]."""
    slots = np.asarray(slots, dtype=np.int64)
    blocks, offsets = slots // 16, slots % 16
    layers = key.shape[0]
    pool[layer_begin : layer_begin + layers, 0, blocks, offsets] = key
    pool[layer_begin : layer_begin + layers, 1, blocks, offsets] = value


def append_rotated(
    pool: np.ndarray,
    key: np.ndarray,
    value: np.ndarray,
    slots: np.ndarray,
    positions: np.ndarray,
    table: np.ndarray,
    layer_begin: int = 0,
) -> None:
    """apply_rope on K at ``positions`` (dense.py:33-61), then the copy."""
    write_rows(pool, layer_begin, rope.rotate(key, positions, table), value, slots)
