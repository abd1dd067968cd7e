"""Oracle of the FP16 RoPE of K and Q (src/pagedcore/dense.py:33-61).

Test infrastructure only.  The cos/sin table is computed by ATen, the
third-party dependency the reference's arithmetic lives in (torch 2.7.1 is
pinned by the reference's uv.lock; torch 2.11 runs here): its FP32 pow/cos/sin
are not correctly rounded, so no independent restatement reproduces every
entry.  ``cos_sin_table`` therefore replays the reference's op sequence
(dense.py:48-54) with torch on the CPU, and the table is pinned against the
golden table extracted from the reference's own apply_rope
(tests/golden/rope_table.npz).  The rotation itself is restated in numpy.
"""

from __future__ import annotations

import numpy as np


def cos_sin_table(context: int = 2048) -> np.ndarray:
    """FP16 [2, context, 32]: cos and sin of position * inverse frequency."""
    import torch

    with torch.autocast(device_type="cpu", enabled=False):
        inverse = 1.0 / (10000.0 ** (torch.arange(0, 64, 2).float() / 64))
        angles = torch.arange(context)[None].float().unsqueeze(-1) * inverse
        angles = torch.cat((angles, angles), dim=-1)
        cos = angles.cos().to(torch.float16)[0, :, :32]
        sin = angles.sin().to(torch.float16)[0, :, :32]
    return np.stack((cos.numpy(), sin.numpy()))


def _round_mul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return (a.astype(np.float32) * b.astype(np.float32)).astype(np.float16)


def _round_add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return (a.astype(np.float32) + b.astype(np.float32)).astype(np.float16)


def rotate(x: np.ndarray, positions: np.ndarray, table: np.ndarray) -> np.ndarray:
    """Rotate FP16 x [..., T, heads, 64] at int positions [T] (dense.py:56-59).

    x*cos + cat(-x[32:], x[:32])*sin with each product and the sum rounded to
    FP16, cos/sin being the FP16 table rows of the positions.
    """
    positions = np.asarray(positions)
    cos = np.concatenate([table[0][positions]] * 2, axis=-1)[:, None, :]  # [T, 1, 64]
    sin = np.concatenate([table[1][positions]] * 2, axis=-1)[:, None, :]
    rotated = np.concatenate((-x[..., 32:], x[..., :32]), axis=-1)
    return _round_add(_round_mul(x, cos), _round_mul(rotated, sin))
