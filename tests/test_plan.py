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
    assert plan.workspace_bytes == (9 + plan.grid) * _PARTIAL_BYTES + plan.grid * 16 + 2048
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
    assert plan.workspace_bytes == (batch + plan.grid) * _PARTIAL_BYTES + plan.grid * 16 + 2048
    big, tail = plan.pieces()
    assert 1 <= big <= plan.grid and tail >= 1


# -- piece tables (pkv_decode_tables, host) ---------------------------------------
def random_prefix(seed: int, rows: int, max_blocks: int = 130) -> np.ndarray:
    rng = np.random.default_rng(seed)
    blocks = rng.integers(1, max_blocks, size=rows)
    return np.concatenate([[0], np.cumsum(blocks)]).astype(np.int32)


def check_tables(prefix: np.ndarray, pieces: np.ndarray, row_pieces: np.ndarray) -> None:
    total, grid = int(prefix[-1]), len(pieces)
    begins, ends = pieces[:, 0], pieces[:, 1]
    assert begins[0] == 0 and ends[-1] == total
    assert np.all(ends > begins) and np.array_equal(begins[1:], ends[:-1])
    rows = np.searchsorted(prefix, begins, side="right") - 1
    assert np.array_equal(pieces[:, 2], rows)
    assert np.array_equal(pieces[:, 3], prefix[rows])
    piece_of = np.searchsorted(begins, np.arange(total), side="right") - 1
    assert np.array_equal(row_pieces[:, 0], piece_of[prefix[:-1]])
    assert np.array_equal(row_pieces[:, 1], piece_of[prefix[1:] - 1])
    assert row_pieces.shape == (len(prefix) - 1, 2) and grid >= 1


def piece_costs(prefix: np.ndarray, pieces: np.ndarray, row_cost: float) -> np.ndarray:
    starts = prefix[1:-1]
    inside = [np.count_nonzero((starts >= b) & (starts < e)) for b, e in pieces[:, :2]]
    return (pieces[:, 1] - pieces[:, 0]) + row_cost * np.asarray(inside)


@pytest.mark.parametrize("rows, grid", [(1, 1), (1, 7), (5, 5), (40, 13), (256, 444), (64, 2000)])
def test_tables_cover_the_blocks_and_index_rows_and_pieces(rows: int, grid: int) -> None:
    prefix = random_prefix(rows, rows)
    grid = min(grid, int(prefix[-1]))
    for row_cost in (0.0, 1.5, 8.0):
        pieces, row_pieces = kernels.decode_tables(prefix, grid, row_cost=row_cost)
        check_tables(prefix, pieces, row_pieces)


def test_tables_balance_blocks_plus_row_switches() -> None:
    prefix = random_prefix(3, 256)
    grid = 444
    plain, _ = kernels.decode_tables(prefix, grid, row_cost=0.0)
    sizes = plain[:, 1] - plain[:, 0]
    assert sizes.max() - sizes.min() <= 1
    costed, _ = kernels.decode_tables(prefix, grid, row_cost=2.0)
    costs = piece_costs(prefix, costed, 2.0)
    assert costs.max() - costs.min() <= 1 + 2.0 * 2  # one block plus the switches at a cut's edges


def test_tables_follow_the_weights() -> None:
    prefix = random_prefix(4, 200)
    grid = 100
    weights = np.where(np.arange(grid) % 2 == 0, 1.0, 1.5).astype(np.float32)
    pieces, row_pieces = kernels.decode_tables(prefix, grid, weights=weights, row_cost=0.0)
    check_tables(prefix, pieces, row_pieces)
    sizes = (pieces[:, 1] - pieces[:, 0]).astype(float)
    ratio = sizes[1::2].mean() / sizes[0::2].mean()
    assert 1.45 < ratio < 1.55
    again = kernels.decode_tables(prefix, grid, weights=weights, row_cost=0.0)
    assert np.array_equal(again[0], pieces) and np.array_equal(again[1], row_pieces)


def test_padded_tables_put_every_region_at_its_fixed_offset() -> None:
    from pagedcore_b200.kv_cache import padded_tables

    lengths = np.array([5, 40, 17], dtype=np.int32)
    prefix = np.concatenate(([0], np.cumsum((lengths + 15) // 16))).astype(np.int32)
    total = int(prefix[-1])
    flat = np.arange(100, 100 + total, dtype=np.int32)
    pieces, row_pieces = kernels.decode_tables(prefix, 2)
    rows, grid = 8, 6
    tables = padded_tables(pieces, row_pieces, np.concatenate((lengths, prefix, flat)), 3, total, rows, grid)
    assert len(tables) == 4 * grid + 4 * rows + 1 + total
    assert np.array_equal(tables[:8].reshape(2, 4), pieces) and not tables[8 : 4 * grid].any()  # empty pieces
    at = 4 * grid
    padded_rows = tables[at : at + 2 * rows].reshape(rows, 2)
    assert np.array_equal(padded_rows[:3], row_pieces) and not padded_rows[3:].any()  # rows with no pieces
    at += 2 * rows
    assert tables[at : at + rows].tolist() == [5, 40, 17, 0, 0, 0, 0, 0]
    at += rows
    assert tables[at : at + rows + 1].tolist() == prefix.tolist() + [total] * (rows - 3)
    assert np.array_equal(tables[at + rows + 1 :], flat)
    with pytest.raises(ValueError, match="layout has 2 and 6"):
        padded_tables(pieces, row_pieces, np.concatenate((lengths, prefix, flat)), 3, total, 2, grid)


def test_tables_reject_bad_arguments() -> None:
    prefix = random_prefix(5, 4, max_blocks=3)
    with pytest.raises(ValueError, match="grid must lie"):
        kernels.decode_tables(prefix, int(prefix[-1]) + 1)
    with pytest.raises(ValueError, match="at least one block"):
        kernels.decode_tables(np.array([0, 2, 2, 5], dtype=np.int32), 2)
    with pytest.raises(ValueError, match="weights must be finite and positive"):
        kernels.decode_tables(prefix, 2, weights=np.array([1.0, 0.0], dtype=np.float32))
    with pytest.raises(ValueError, match="row_cost"):
        kernels.decode_tables(prefix, 2, row_cost=-1.0)


@pytest.mark.gpu
@pytest.mark.parametrize("grid, row_cost, seed", [(7, 0.0, 1), (40, 1.5, 2), (271, 4.0, 3)])
def test_any_piece_tables_give_the_reference_attention(grid: int, row_cost: float, seed: int) -> None:
    import torch

    from pagedcore_b200 import workloads
    from tests.test_attention_gpu import build_batch, oracle_rows

    device = cuda_device()
    lengths = [1, 16, 17, 33, 250, 700, 2048, 5, 1200]
    allocator, requests = build_batch(lengths, 33, device)
    query = torch.from_numpy(workloads.normal_f16(workloads.rng(33, 8), (len(lengths), 32, 64))).to(device)
    batch = allocator.decode_batch(requests, layer_index=4)
    prefix = batch.prefix.cpu().numpy()
    weights = np.random.default_rng(seed).uniform(0.5, 2.0, grid).astype(np.float32)
    pieces, row_pieces = kernels.decode_tables(prefix, grid, weights=weights, row_cost=row_cost)
    # With tables the partition arguments are ignored; only the grid matters.
    plan = kernels.DecodePlan(grid, 1, kernels.workspace_bytes(len(lengths), grid))
    workspace = torch.zeros(plan.workspace_bytes // 4, dtype=torch.float32, device=device)
    out = torch.empty_like(query)
    kernels.decode_attention(allocator.pool, 4, query, batch.lengths, batch.prefix, batch.flat, batch.total_blocks,
                             plan, out, workspace, allocator._error,
                             torch.from_numpy(pieces).to(device), torch.from_numpy(row_pieces).to(device))
    expected = oracle_rows(allocator, requests, query, 4, range(len(lengths)))
    for row in range(len(lengths)):
        np.testing.assert_allclose(out[row].cpu().numpy().astype(np.float32), expected[row].astype(np.float32),
                                   atol=2e-3, rtol=1e-2)
    allocator.check_device_errors()


@pytest.mark.gpu
def test_measured_balance_learns_weights_and_matches_the_row_balanced_cut() -> None:
    import torch

    from pagedcore_b200 import workloads
    from pagedcore_b200.engine_types import KVReservation, RequestId
    from pagedcore_b200.kv_cache import KVAllocator

    device = cuda_device()
    lengths = workloads.decode_lengths(12, 96, high=1900).tolist()
    need = sum(-(-(n + 20) // 16) for n in lengths) + 8
    requests = tuple(RequestId(f"m{i}") for i in range(len(lengths)))
    allocators = []
    for balance in ("rows", "measured"):
        pool = torch.empty((22, 2, need, 16, 4, 64), dtype=torch.float16, device=device)
        allocator = KVAllocator(pool, validation="incremental", balance=balance)
        generator = torch.Generator(device=device).manual_seed(12)
        for request, length in zip(requests, lengths, strict=True):
            allocator.create(KVReservation(request, -(-(length + 20) // 16)))
            kv = torch.randn(22, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
            allocator.append(request, kv, kv)
        allocators.append(allocator)
    rows, measured = allocators
    generator = torch.Generator(device=device).manual_seed(13)
    q = torch.randn(len(lengths), 32, 64, dtype=torch.float16, device=device, generator=generator)
    k = torch.randn(len(lengths), 4, 64, dtype=torch.float16, device=device, generator=generator)
    frozen = None
    for step in range(14):
        outs = []
        for allocator in allocators:
            with allocator.append_decode(requests):
                outs.append([allocator.decode_layer(layer, q, k, k) for layer in (range(22))])
        for a, b in zip(*outs, strict=True):
            torch.testing.assert_close(b, a, atol=2e-3, rtol=1e-2)
        if step == 9:
            frozen = measured.slot_weights()
    weights = measured.slot_weights()
    (grid, w), = weights.items()
    assert measured._speeds[grid].updates == 6
    assert np.array_equal(w, frozen[grid])  # frozen: the cut no longer changes
    assert abs(float(w.mean()) - 1.0) < 1e-3 and 0.5 <= w.min() and w.max() <= 2.0
    assert rows.slot_weights() == {}
    for allocator in allocators:
        allocator.check_device_errors()
