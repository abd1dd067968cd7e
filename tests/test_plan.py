"""Split plans of the decode attention: pieces cover the flat block list exactly."""

from __future__ import annotations

import numpy as np
import pytest

from pagedcore_b200 import kernels
from tests.conftest import cuda_device

_PARTIAL_BYTES = 32 * 66 * 4


def piece_ends(plan: kernels.DecodePlan, total: int) -> np.ndarray:
    starts = plan.piece_starts()
    return np.minimum(np.append(starts[1:], total), total)


@pytest.mark.parametrize(
    "total, pieces",
    [(1, (1, 0, 0)), (271, (5, 0, 0)), (271, (1000, 0, 0)), (271, (20, 10, 3)), (271, (7, 30, 1)), (306, (100, 2, 5))],
)
def test_pieces_are_contiguous_nonempty_and_cover_every_block(total: int, pieces: tuple[int, int, int]) -> None:
    plan = kernels.DecodePlan.split(9, total, *pieces)
    starts = plan.piece_starts()
    ends = piece_ends(plan, total)
    assert starts[0] == 0 and ends[-1] == total
    assert np.all(ends > starts)
    assert np.array_equal(starts[1:], ends[:-1])
    assert plan.workspace_bytes == (9 + plan.grid) * _PARTIAL_BYTES
    big, tail = plan.pieces()
    sizes = ends - starts
    full = sizes[:-1]  # every piece but the last has its nominal size
    assert np.all(full[:big] == plan.blocks_per_cta)
    assert np.all(full[big:] == tail)


@pytest.mark.gpu
@pytest.mark.parametrize("batch, total", [(1, 1), (4, 300), (256, 14142), (1024, 131072)])
def test_device_plan_is_a_valid_partition(batch: int, total: int) -> None:
    device = cuda_device()
    plan = kernels.decode_plan(device, batch, total)
    starts = plan.piece_starts()
    ends = piece_ends(plan, total)
    assert starts[0] == 0 and ends[-1] == total and np.all(ends > starts)
    assert plan.workspace_bytes == (batch + plan.grid) * _PARTIAL_BYTES
    big, tail = plan.pieces()
    assert 1 <= big <= plan.grid and tail >= 1
