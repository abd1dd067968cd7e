"""Split-K decode attention on the GPU against the reference, the oracle and FP64.

Tolerances are the reference's own (docs/NUMERICAL_POLICY.md:24 and
tests/unit/test_attention.py): atol 2e-3 / rtol 2e-3 against the FP64 dense
oracle, and BASELINE's max-abs 2e-3 / rel 1e-2 against the reference's FP32
paged_attention; the analytic known answers of the reference tests are exact.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oracle_attention
from pagedcore_b200 import kernels, workloads
from pagedcore_b200.attention import paged_attention, paged_decode_attention
from pagedcore_b200.engine_types import CapacityCounts, KVReservation, RequestId
from pagedcore_b200.kv_cache import KVAllocator
from tests.conftest import cuda_device

pytestmark = pytest.mark.gpu


def dense_reference(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> torch.Tensor:
    """FP64 per-head oracle (tests/unit/test_attention.py:173-179); query [1,32,1,64], key/value [L,4,64]."""
    out = oracle_attention.dense_fp64(
        query.detach().reshape(32, 64).cpu().numpy(), key.cpu().numpy(), value.cpu().numpy()
    )
    return torch.from_numpy(out).reshape(1, 32, 1, 64)


def poisoned_cache(key: torch.Tensor, value: torch.Tensor) -> tuple[KVAllocator, RequestId, torch.Tensor]:
    """NaN pool with sentinel blockers so the request's table is fragmented
    (tests/gpu/test_attention_cuda.py:93-125)."""
    device = key.device
    tokens = key.shape[1]
    blocks = (tokens + 15) // 16
    pool = torch.full((22, 2, blocks + 3, 16, 4, 64), torch.nan, dtype=torch.float16, device=device)
    allocator = KVAllocator(pool)
    for name in ("first", "retained", "last"):
        request = RequestId(name)
        allocator.create(KVReservation(request, 1))
        sentinel = torch.full((22, 16, 4, 64), -100.0, dtype=torch.float16, device=device)
        allocator.append(request, sentinel, -sentinel)
    allocator.release_all(RequestId("first"))
    allocator.release_all(RequestId("last"))
    request = RequestId("attention")
    allocator.create(KVReservation(request, blocks))
    allocator.append(request, key, value)
    table = allocator.block_table(request)
    if blocks > 1:
        assert table != tuple(range(table[0], table[0] + blocks))
    return allocator, request, pool


def check_attention(query, key, value, *, layer: int, atol: float = 2e-3) -> None:
    allocator, request, pool = poisoned_cache(key, value)
    before = pool.clone()
    counts = allocator.capacity()
    table = allocator.block_table(request)
    actual = paged_attention(query, allocator, request, layer_index=layer)
    with torch.autocast("cuda", dtype=torch.float16):
        autocast_actual = paged_attention(query, allocator, request, layer_index=layer)
    torch.cuda.synchronize()
    allocator.check_device_errors()
    expected = dense_reference(query, key[layer], value[layer])
    assert actual.shape == (1, 32, 1, 64) and actual.dtype == torch.float16
    assert actual.device == query.device and not actual.requires_grad
    assert torch.isfinite(actual).all()
    torch.testing.assert_close(actual.cpu(), expected, atol=atol, rtol=2e-3)
    assert torch.equal(autocast_actual, actual)
    torch.testing.assert_close(pool, before, atol=0, rtol=0, equal_nan=True)
    assert allocator.block_table(request) == table and allocator.capacity() == counts


@pytest.mark.parametrize("tokens,layer", [(1, 0), (15, 21), (16, 7), (17, 0), (49, 21), (2048, 11)])
def test_boundaries_match_fp64(tokens: int, layer: int) -> None:
    # tests/gpu/test_attention_cuda.py:148-157
    device = cuda_device()
    generator = torch.Generator(device=device).manual_seed(tokens * 31 + layer)
    key = torch.randn(22, tokens, 4, 64, dtype=torch.float16, device=device, generator=generator)
    value = torch.randn(22, tokens, 4, 64, dtype=torch.float16, device=device, generator=generator)
    query = torch.randn(1, 32, 1, 128, dtype=torch.float16, device=device, generator=generator)
    check_attention(query[..., ::2].requires_grad_(), key, value, layer=layer)


def test_gqa_maps_eight_query_heads_per_kv_head() -> None:
    # tests/unit/test_attention.py:281-302: exact 100*(h//8)+16
    device = cuda_device()
    key = torch.zeros(22, 33, 4, 64, dtype=torch.float16, device=device)
    values = 100 * torch.arange(4, device=device)[None, :] + torch.arange(33, device=device)[:, None]
    value = values[None, :, :, None].expand(22, 33, 4, 64).half().contiguous()
    allocator, request, _ = poisoned_cache(key, value)
    actual = paged_attention(torch.zeros(1, 32, 1, 64, dtype=torch.float16, device=device), allocator, request,
                             layer_index=21)
    for head in range(32):
        assert torch.equal(actual[0, head, 0].cpu(), torch.full((64,), 100 * (head // 8) + 16).half())


def test_normalizes_all_scores_before_value_products() -> None:
    # tests/unit/test_attention.py:182-221: 16 tokens of 2 and one of 19 -> exactly 3
    device = cuda_device()
    key = torch.zeros(22, 17, 4, 64, dtype=torch.float16, device=device)
    value = torch.zeros_like(key)
    value[:, :16], value[:, 16:] = 2, 19
    allocator, request, _ = poisoned_cache(key, value)
    actual = paged_attention(torch.zeros(1, 32, 1, 64, dtype=torch.float16, device=device), allocator, request,
                             layer_index=0)
    assert torch.equal(actual, torch.full_like(actual, 3))


def test_tiny_probabilities_survive_until_value_accumulation() -> None:
    # tests/unit/test_attention.py:224-242: exp(-20) weights remain visible
    device = cuda_device()
    key = torch.zeros(22, 17, 4, 64, dtype=torch.float16, device=device)
    key[:, :, :, 0] = -160
    key[:, 0, :, 0] = 0
    value = torch.full_like(key, 65504)
    value[:, 0] = 0
    query = torch.zeros(1, 32, 1, 64, dtype=torch.float16, device=device)
    query[..., 0] = 1
    allocator, request, _ = poisoned_cache(key, value)
    actual = paged_attention(query, allocator, request, layer_index=0)
    assert (actual > 0).all()
    torch.testing.assert_close(actual.cpu(), dense_reference(query, key[0], value[0]), atol=1e-6, rtol=2e-3)


def test_rounds_only_after_cancellation_across_pages() -> None:
    # tests/unit/test_attention.py:245-259: exactly 0.25
    device = cuda_device()
    key = torch.zeros(22, 32, 4, 64, dtype=torch.float16, device=device)
    value = torch.zeros_like(key)
    value[:, 0], value[:, 1], value[:, 16] = 32768, 8, -32768
    allocator, request, _ = poisoned_cache(key, value)
    actual = paged_attention(torch.zeros(1, 32, 1, 64, dtype=torch.float16, device=device), allocator, request,
                             layer_index=0)
    assert torch.equal(actual, torch.full_like(actual, 0.25))


@pytest.mark.parametrize("reverse", [False, True])
@pytest.mark.parametrize("query_scale", [1.0, 1000.0])
def test_rescales_softmax_across_large_block_scores(reverse: bool, query_scale: float) -> None:
    # tests/unit/test_attention.py:305-322
    device = cuda_device()
    key = torch.full((22, 49, 4, 64), -1000.0, dtype=torch.float16, device=device)
    key[:, 16:32] = 0
    key[:, 32:] = 1000
    generator = torch.Generator(device=device).manual_seed(int(query_scale) + reverse)
    value = torch.randn(key.shape, dtype=torch.float16, device=device, generator=generator)
    if reverse:
        key, value = key.flip(1).contiguous(), value.flip(1).contiguous()
    query = torch.full((1, 32, 1, 64), query_scale, dtype=torch.float16, device=device)
    check_attention(query, key, value, layer=0)


@pytest.mark.parametrize("state", ["unknown", "empty", "released"])
def test_rejects_requests_without_cached_tokens(state: str) -> None:
    device = cuda_device()
    allocator = KVAllocator(torch.empty(22, 2, 1, 16, 4, 64, dtype=torch.float16, device=device))
    request = RequestId("missing")
    if state != "unknown":
        allocator.create(KVReservation(request, 1))
    if state == "released":
        allocator.release_all(request)
    before = allocator.capacity()
    with pytest.raises(ValueError if state == "empty" else KeyError):
        paged_attention(torch.zeros(1, 32, 1, 64, dtype=torch.float16, device=device), allocator, request,
                        layer_index=0)
    assert allocator.capacity() == before


def test_rejects_invalid_queries_layers_and_devices() -> None:
    device = cuda_device()
    key = torch.zeros(22, 1, 4, 64, dtype=torch.float16, device=device)
    allocator, request, _ = poisoned_cache(key, key)
    for query in (torch.zeros(2, 32, 1, 64), torch.zeros(1, 31, 1, 64), torch.zeros(1, 32, 2, 64),
                  torch.zeros(1, 32, 1, 63)):
        with pytest.raises(ValueError, match="query must be FP16"):
            paged_attention(query.half().to(device), allocator, request, layer_index=0)
    with pytest.raises(ValueError, match="query must be FP16"):
        paged_attention(torch.zeros(1, 32, 1, 64, device=device), allocator, request, layer_index=0)
    for layer in (-1, 22, True, 1.0):
        with pytest.raises(ValueError, match="layer_index"):
            paged_attention(torch.zeros(1, 32, 1, 64, dtype=torch.float16, device=device), allocator, request,
                            layer_index=layer)
    with pytest.raises(ValueError, match="same device"):
        paged_attention(torch.zeros(1, 32, 1, 64, dtype=torch.float16), allocator, request, layer_index=0)


def build_batch(lengths, seed: int, device: torch.device, room: int = 0) -> tuple[KVAllocator, tuple]:
    need = sum(workloads.blocks_for(n + room) for n in lengths) + 8
    pool = torch.full((22, 2, need, 16, 4, 64), torch.nan, dtype=torch.float16, device=device)
    allocator = KVAllocator(pool, validation="incremental")
    order = workloads.rng(seed, 7).permutation(need).astype(np.int32)
    allocator.ledger.reorder_free(order)
    generator = torch.Generator(device=device).manual_seed(seed)
    requests = []
    for row, length in enumerate(lengths):
        request = RequestId(f"r{row}")
        allocator.create(KVReservation(request, workloads.blocks_for(length + room)))
        key = torch.randn(22, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
        value = torch.randn(22, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
        allocator.append(request, key, value)
        requests.append(request)
    return allocator, tuple(requests)


def oracle_rows(allocator: KVAllocator, requests, query: torch.Tensor, layer: int, rows) -> list[np.ndarray]:
    pool_layer = allocator.pool[layer : layer + 1].cpu().numpy()
    q = query.cpu().numpy()
    outputs = []
    for row in rows:
        blocks = allocator.block_table(requests[row])
        length = allocator.cached_length(requests[row])
        outputs.append(oracle_attention.paged_attention(pool_layer, 0, q[row], blocks, length))
    return outputs


def test_config1_matches_reference_outputs(attention_golden: dict) -> None:
    device = cuda_device()
    case = workloads.attention_case()
    pool = torch.full((22, 2, case.num_blocks, 16, 4, 64), torch.nan, dtype=torch.float16, device=device)
    allocator = KVAllocator(pool)
    allocator.ledger.reorder_free(case.free_order)
    requests = tuple(RequestId(f"row{i}") for i in range(len(case.lengths)))
    for request, length, key, value in zip(requests, case.lengths, case.keys, case.values, strict=True):
        allocator.create(KVReservation(request, workloads.blocks_for(length)))
        allocator.append(request, torch.from_numpy(key).to(device), torch.from_numpy(value).to(device))
    flat = np.concatenate([np.asarray(allocator.block_table(r), dtype=np.int32) for r in requests])
    assert np.array_equal(flat, attention_golden["tables"])
    query = torch.from_numpy(case.query).to(device)
    for layer in (0, 21):
        batched = paged_decode_attention(query, allocator, requests, layer_index=layer).cpu().float()
        reference = torch.from_numpy(attention_golden[f"out_layer{layer}"]).float()
        dense = torch.from_numpy(attention_golden[f"dense_layer{layer}"]).float()
        torch.testing.assert_close(batched, reference, atol=2e-3, rtol=1e-2)
        torch.testing.assert_close(batched, dense, atol=2e-3, rtol=2e-3)
        for row, request in enumerate(requests):
            single = paged_attention(query[row].reshape(1, 32, 1, 64), allocator, request, layer_index=layer)
            torch.testing.assert_close(single.reshape(32, 64).cpu().float(), reference[row], atol=2e-3, rtol=1e-2)
    allocator.check_device_errors()


def test_ragged_batch_matches_oracle() -> None:
    device = cuda_device()
    lengths = workloads.decode_lengths(21, 96, high=2048).tolist()
    allocator, requests = build_batch(lengths, 21, device)
    query = torch.from_numpy(workloads.normal_f16(workloads.rng(21, 8), (len(lengths), 32, 64))).to(device)
    for layer in (0, 13):
        out = paged_decode_attention(query, allocator, requests, layer_index=layer).cpu().numpy()
        rows = range(0, len(lengths), 5)
        for row, expected in zip(rows, oracle_rows(allocator, requests, query, layer, rows), strict=True):
            np.testing.assert_allclose(out[row].astype(np.float32), expected.astype(np.float32), atol=2e-3, rtol=1e-2)
    allocator.check_device_errors()


# (blocks_per_cta, big_ctas, tail_blocks): uniform splits (big_ctas 0) and
# two-tier splits, big pieces followed by tail pieces.
@pytest.mark.parametrize("pieces", [(1, 0, 0), (2, 0, 0), (3, 0, 0), (5, 0, 0), (8, 0, 0), (64, 0, 0), (1000, 0, 0), (20, 10, 3), (7, 30, 1), (100, 2, 5)])
def test_every_split_plan_gives_the_same_answer(pieces: tuple[int, int, int]) -> None:
    device = cuda_device()
    lengths = [1, 16, 17, 33, 250, 700, 2048, 5, 1200]
    allocator, requests = build_batch(lengths, 33, device)
    query = torch.from_numpy(workloads.normal_f16(workloads.rng(33, 8), (len(lengths), 32, 64))).to(device)
    batch = allocator.decode_batch(requests, layer_index=4)
    plan = kernels.DecodePlan.split(len(lengths), batch.total_blocks, *pieces)
    workspace = torch.zeros(plan.workspace_bytes // 4, dtype=torch.float32, device=device)
    out = torch.empty_like(query)
    kernels.decode_attention(allocator.pool, 4, query, batch.lengths, batch.prefix, batch.flat, batch.total_blocks,
                             plan, out, workspace, allocator._error)
    expected = oracle_rows(allocator, requests, query, 4, range(len(lengths)))
    for row in range(len(lengths)):
        np.testing.assert_allclose(out[row].cpu().numpy().astype(np.float32), expected[row].astype(np.float32),
                                   atol=2e-3, rtol=1e-2)
    allocator.check_device_errors()


def test_decode_attends_the_token_written_in_the_same_step() -> None:
    # decoder.py:187-190: write before read, so the current token is attended.
    device = cuda_device()
    allocator, requests = build_batch([15, 16, 40], 44, device, room=1)
    count = len(requests)
    key = torch.zeros(22, count, 4, 64, dtype=torch.float16, device=device)
    value = torch.full((22, count, 4, 64), 7.0, dtype=torch.float16, device=device)
    # A huge score on the new token makes the output equal its value.
    query = torch.zeros(count, 32, 64, dtype=torch.float16, device=device)
    with allocator.append_decode(requests):
        for layer in range(22):
            k = key[layer].clone()
            k[..., 0] = 1000
            q = query.clone()
            q[..., 0] = 1000
            allocator.write_decode_batch(layer, k, value[layer])
            out = paged_decode_attention(q, allocator, requests, layer_index=layer)
            torch.testing.assert_close(out, torch.full_like(out, 7.0), atol=0, rtol=0)
    assert [allocator.cached_length(r) for r in requests] == [16, 17, 41]
    counts = allocator.capacity()
    assert (counts.owned_blocks, counts.reserved_blocks, counts.live_cached_token_slots) == (6, 6, 74)
    assert isinstance(counts, CapacityCounts)
