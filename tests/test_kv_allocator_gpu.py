"""KV writes on the GPU: bit-exact against the reference's golden pools and the oracle.

Also ports the data-carrying allocator tests of the reference
(tests/unit/test_kv_cache.py, tests/gpu/test_kv_pool_cuda.py) to CUDA pools.
"""

from __future__ import annotations

import hashlib
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest
import torch

from oracle import kv_write
from oracle.allocator import OracleAllocator
from pagedcore_b200 import kernels as kernels_module
from pagedcore_b200 import workloads
from pagedcore_b200.engine_types import CapacityCounts, KVReservation, RequestId
from pagedcore_b200.kv_cache import KVAllocator
from tests.conftest import SMALL_CASE, cuda_device

pytestmark = pytest.mark.gpu


def sha256(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).view(np.uint8)).hexdigest()


def nan_pool(blocks: int, device: torch.device) -> torch.Tensor:
    return torch.full((22, 2, blocks, 16, 4, 64), torch.nan, dtype=torch.float16, device=device)


def kv_values(tokens: int, start: float = 0, device: torch.device | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    key = torch.arange(22 * tokens * 4 * 64, dtype=torch.float32).reshape(22, tokens, 4, 64)
    key = (key / 256 + start).half().to(device)
    return key, -key - 1


def replay(allocator: KVAllocator, case: workloads.AppendCase, device: torch.device, checkpoints: dict | None = None):
    pool = allocator.pool
    for index, op in enumerate(case.churn):
        rid = RequestId(str(op.request))
        if op.kind == "create":
            allocator.create(KVReservation(rid, op.credits))
            key, value = workloads.churn_fill(index, op.tokens)
            allocator.append(rid, torch.from_numpy(key).to(device), torch.from_numpy(value).to(device))
        else:
            allocator.release_all(rid)
    if checkpoints is not None:
        checkpoints["after_churn"] = (allocator.capacity(), sha256(pool.cpu().numpy()))
    for prompt in case.prompts:
        rid = RequestId(str(prompt.request))
        allocator.create(KVReservation(rid, prompt.credits))
        allocator.append(rid, torch.from_numpy(prompt.key).to(device), torch.from_numpy(prompt.value).to(device),
                         rotate=True)
    if checkpoints is not None:
        checkpoints["after_prompts"] = (allocator.capacity(), sha256(pool.cpu().numpy()))
    requests = tuple(RequestId(str(r)) for r in case.decode.requests)
    key = torch.from_numpy(case.decode.key).to(device)
    value = torch.from_numpy(case.decode.value).to(device)
    with allocator.append_decode(requests):
        for layer in range(22):
            allocator.write_decode_batch(layer, key[layer], value[layer], rotate=True)
    allocator.check_device_errors()
    return requests


def test_small_append_case_is_bit_exact(append_small_golden: dict, rope_golden: np.ndarray) -> None:
    device = cuda_device()
    case = workloads.append_case(**SMALL_CASE)
    allocator = KVAllocator(nan_pool(case.num_blocks, device))
    replay(allocator, case, device)
    pool = allocator.pool.cpu().numpy()
    assert sha256(pool) == bytes(append_small_golden["pool_sha256"]).hex()
    assert np.array_equal(pool[0].view(np.uint16), append_small_golden["pool_layer0"].view(np.uint16))
    counts = allocator.capacity()
    assert [counts.total_blocks, counts.free_blocks, counts.owned_blocks, counts.reserved_blocks,
            counts.active_slots, counts.live_cached_token_slots] == append_small_golden["capacity"].tolist()
    assert allocator.ledger.free_list() == append_small_golden["free_list"].tolist()
    # And against the oracle, byte for byte.
    from tests.test_oracle_golden import replay_append

    oracle_pool, _, _ = replay_append(case, rope_golden)
    assert np.array_equal(pool.view(np.uint16), oracle_pool.view(np.uint16))


def test_config2_append_matches_reference_pool(append_golden: dict) -> None:
    """Config 2 at full size: 4096 blocks, 10k churn ops, 8 prompts, 256 decode rows."""
    device = cuda_device()
    case = workloads.append_case()
    allocator = KVAllocator(nan_pool(case.num_blocks, device), validation="incremental")
    checkpoints: dict = {}
    requests = replay(allocator, case, device, checkpoints)
    for name in ("after_churn", "after_prompts"):
        counts, digest = checkpoints[name]
        assert digest == append_golden[name]["pool_sha256"], name
        assert [counts.total_blocks, counts.free_blocks, counts.owned_blocks, counts.reserved_blocks,
                counts.active_slots, counts.live_cached_token_slots] == append_golden[name]["capacity"]
    assert sha256(allocator.pool.cpu().numpy()) == append_golden["after_decode"]["pool_sha256"]
    for request in requests:
        assert list(allocator.block_table(request)) == append_golden["after_decode"]["tables"][request]


def test_config2_prompts_in_one_batched_append_match_reference_pool(append_golden: dict) -> None:
    """append_many of config 2's 8 prompts in one launch gives the reference's pool bytes."""
    device = cuda_device()
    case = workloads.append_case()
    allocator = KVAllocator(nan_pool(case.num_blocks, device), validation="incremental")
    for index, op in enumerate(case.churn):
        rid = RequestId(str(op.request))
        if op.kind == "create":
            allocator.create(KVReservation(rid, op.credits))
            key, value = workloads.churn_fill(index, op.tokens)
            allocator.append(rid, torch.from_numpy(key).to(device), torch.from_numpy(value).to(device))
        else:
            allocator.release_all(rid)
    requests = [RequestId(str(prompt.request)) for prompt in case.prompts]
    for request, prompt in zip(requests, case.prompts, strict=True):
        allocator.create(KVReservation(request, prompt.credits))
    key = torch.from_numpy(np.concatenate([p.key for p in case.prompts], axis=1)).to(device)
    value = torch.from_numpy(np.concatenate([p.value for p in case.prompts], axis=1)).to(device)
    allocator.append_many(requests, key, value, [p.key.shape[1] for p in case.prompts], rotate=True)
    counts = allocator.capacity()
    assert sha256(allocator.pool.cpu().numpy()) == append_golden["after_prompts"]["pool_sha256"]
    assert [counts.total_blocks, counts.free_blocks, counts.owned_blocks, counts.reserved_blocks,
            counts.active_slots, counts.live_cached_token_slots] == append_golden["after_prompts"]["capacity"]
    allocator.check_device_errors()


def test_a_failing_batched_append_writes_and_publishes_nothing() -> None:
    device = cuda_device()
    allocator = KVAllocator(nan_pool(8, device))
    allocator.create(KVReservation(RequestId("a"), 2))
    allocator.create(KVReservation(RequestId("b"), 1))
    key, value = kv_values(40, device=device)
    counts = allocator.capacity()
    with pytest.raises(RuntimeError, match="exceeds request reservation"):  # b holds 16 positions
        allocator.append_many([RequestId("a"), RequestId("b")], key, value, [20, 20])
    with pytest.raises(KeyError):
        allocator.append_many([RequestId("a"), RequestId("zz")], key, value, [20, 20])
    with pytest.raises(ValueError, match="sum"):
        allocator.append_many([RequestId("a"), RequestId("b")], key, value, [20, 10])
    assert allocator.capacity() == counts
    assert torch.isnan(allocator.pool).all()
    allocator.append_many([RequestId("a"), RequestId("b")], key[:, :30], value[:, :30], [20, 10])
    assert allocator.cached_length(RequestId("a")) == 20 and allocator.cached_length(RequestId("b")) == 10


def test_per_row_and_batched_decode_writes_agree(rope_golden: np.ndarray) -> None:
    device = cuda_device()
    lengths = [1, 15, 16, 17, 31, 32, 100]
    pools = [nan_pool(64, device) for _ in range(2)]
    allocators = [KVAllocator(pool) for pool in pools]
    generator = workloads.rng(3, 9)
    for allocator in allocators:
        for row, length in enumerate(lengths):
            allocator.create(KVReservation(RequestId(str(row)), workloads.blocks_for(length + 1)))
            key = torch.from_numpy(workloads.normal_f16(workloads.rng(3, row), (22, length, 4, 64))).to(device)
            allocator.append(RequestId(str(row)), key, -key)
    requests = tuple(RequestId(str(row)) for row in reversed(range(len(lengths))))
    key = torch.from_numpy(workloads.normal_f16(generator, (22, len(lengths), 4, 64))).to(device)
    value = torch.from_numpy(workloads.normal_f16(generator, (22, len(lengths), 4, 64))).to(device)
    # Per-row writes take already-rotated K, as write_decode_layer does in the reference.
    positions = np.array([lengths[int(r)] for r in requests])
    from oracle import rope

    rotated = torch.from_numpy(rope.rotate(key.cpu().numpy(), positions, rope_golden)).to(device)
    with allocators[0].append_decode(requests):
        for layer in range(22):
            for row, request in enumerate(requests):
                allocators[0].write_decode_layer(request, layer, rotated[layer, row], value[layer, row])
    with allocators[1].append_decode(requests):
        for layer in range(22):
            allocators[1].write_decode_batch(layer, key[layer], value[layer], rotate=True)
    assert torch.equal(pools[0].view(torch.int16), pools[1].view(torch.int16))
    assert allocators[0].capacity() == allocators[1].capacity()


@pytest.mark.parametrize("tokens,blocks,last_slots", [(1, 1, 1), (15, 1, 15), (16, 1, 16), (17, 2, 1), (32, 2, 16), (33, 3, 1)])
def test_maps_tokens_and_limits_reads_to_valid_slots(tokens: int, blocks: int, last_slots: int) -> None:
    # tests/unit/test_kv_cache.py:150-181 on a CUDA pool
    device = cuda_device()
    pool = nan_pool(4, device)
    allocator = KVAllocator(pool)
    request = RequestId("a")
    allocator.create(KVReservation(request, blocks))
    assert allocator.block_table(request) == () and allocator.cached_length(request) == 0
    key, value = kv_values(tokens, device=device)
    allocator.append(request, key, value)
    table = allocator.block_table(request)
    assert len(table) == blocks and len(set(table)) == blocks
    for index, physical in enumerate(table):
        slots = last_slots if index == blocks - 1 else 16
        actual_key, actual_value = allocator.read_block(request, index)
        assert actual_key.shape == actual_value.shape == (22, slots, 4, 64)
        assert actual_key.untyped_storage().data_ptr() == pool.untyped_storage().data_ptr()
        expected = slice(index * 16, index * 16 + slots)
        assert torch.equal(actual_key, key[:, expected]) and torch.equal(actual_value, value[:, expected])
        if slots < 16:
            assert torch.isnan(pool[:, :, physical, slots:]).all()


def test_fragmented_appends_leave_other_requests_alone() -> None:
    # tests/unit/test_kv_cache.py:184-211
    device = cuda_device()
    allocator = KVAllocator(nan_pool(4, device))
    a, b = RequestId("a"), RequestId("b")
    allocator.create(KVReservation(a, 3))
    allocator.create(KVReservation(b, 1))
    key, value = kv_values(33, device=device)
    other_key, other_value = kv_values(16, start=2000, device=device)
    allocator.append(a, key[:, :15], value[:, :15])
    allocator.append(b, other_key, other_value)
    allocator.append(a, key[:, 15:16], value[:, 15:16])
    allocator.append(a, key[:, 16:17], value[:, 16:17])
    allocator.append(a, key[:, 17:], value[:, 17:])
    assert tuple(allocator.block_table(a)) == (0, 2, 3)
    assert tuple(allocator.block_table(b)) == (1,)
    for index, expected in enumerate((slice(0, 16), slice(16, 32), slice(32, 33))):
        actual_key, actual_value = allocator.read_block(a, index)
        assert torch.equal(actual_key, key[:, expected]) and torch.equal(actual_value, value[:, expected])
    actual_key, actual_value = allocator.read_block(b, 0)
    assert torch.equal(actual_key, other_key) and torch.equal(actual_value, other_value)


def test_release_and_reuse_without_stale_slots() -> None:
    # tests/unit/test_kv_cache.py:214-251
    device = cuda_device()
    pool = torch.empty((22, 2, 3, 16, 4, 64), dtype=torch.float16, device=device)
    allocator = KVAllocator(pool)
    a, b, c = RequestId("a"), RequestId("b"), RequestId("c")
    allocator.create(KVReservation(a, 2))
    allocator.create(KVReservation(b, 1))
    allocator.append(a, *kv_values(17, device=device))
    allocator.append(b, *kv_values(16, start=2000, device=device))
    released = allocator.block_table(a)
    allocator.release_all(a)
    with pytest.raises(KeyError):
        allocator.read_block(a, 0)
    with pytest.raises(KeyError):
        allocator.release_all(a)
    allocator.create(KVReservation(c, 1))
    key, value = kv_values(1, start=-100, device=device)
    allocator.append(c, key, value)
    assert allocator.block_table(c)[0] in released
    actual_key, actual_value = allocator.read_block(c, 0)
    assert actual_key.shape == (22, 1, 4, 64) and torch.equal(actual_key, key) and torch.equal(actual_value, value)
    expected_key, expected_value = kv_values(16, start=2000, device=device)
    assert torch.equal(allocator.read_block(b, 0)[0], expected_key)
    allocator.release_all(b)
    allocator.release_all(c)
    allocator.create(KVReservation(a, 3))
    allocator.append(a, *kv_values(48, device=device))
    assert set(allocator.block_table(a)) == {0, 1, 2}


def test_invalid_appends_and_context_overflow() -> None:
    device = cuda_device()
    allocator = KVAllocator(torch.empty((22, 2, 128, 16, 4, 64), dtype=torch.float16, device=device))
    request = RequestId("a")
    allocator.create(KVReservation(request, 128))
    key, value = kv_values(1, device=device)
    for bad in (value[:1, :, :, :63], value.float(), value.cpu(), value[:, :0]):
        with pytest.raises(ValueError, match="K and V must share"):
            allocator.append(request, key if bad.shape[1] else key[:, :0], bad)
    assert allocator.block_table(request) == () and allocator.cached_length(request) == 0
    allocator.append(request, *kv_values(2048, device=device))
    last = [t.clone() for t in allocator.read_block(request, 127)]
    with pytest.raises(ValueError, match="2048"):
        allocator.append(request, *kv_values(1, device=device))
    assert allocator.cached_length(request) == 2048
    assert all(torch.equal(a, b) for a, b in zip(allocator.read_block(request, 127), last))
    with pytest.raises(KeyError):
        allocator.append(RequestId("missing"), key, value)


def test_decode_append_exposes_only_written_layers_and_commits_together() -> None:
    # tests/unit/test_kv_cache.py:375-418 on a CUDA pool
    device = cuda_device()
    pool = nan_pool(4, device)
    allocator = KVAllocator(pool)
    requests = (RequestId("first"), RequestId("second"))
    for request in requests:
        allocator.create(KVReservation(request, 2))
        allocator.append(request, *kv_values(16, device=device))
    counts = allocator.capacity()
    tables = [allocator.block_table(request) for request in requests]
    key, value = kv_values(1, start=100, device=device)
    with allocator.append_decode(requests):
        with pytest.raises(RuntimeError, match="unwritten"):
            list(allocator.iter_layer_blocks(requests[0], layer_index=0))
        for operation in (
            lambda: allocator.create(KVReservation(RequestId("other"), 1)),
            lambda: allocator.append(requests[0], key, value),
            lambda: allocator.release_all(requests[0]),
            lambda: allocator.append_decode(requests).__enter__(),
        ):
            with pytest.raises(RuntimeError, match="staged decode"):
                operation()
        for layer in range(22):
            for request in requests:
                allocator.write_decode_layer(request, layer, key[layer, 0], value[layer, 0])
                pages = list(allocator.iter_layer_blocks(request, layer_index=layer))
                assert len(pages) == 2
                assert torch.equal(pages[1][0], key[layer]) and torch.equal(pages[1][1], value[layer])
                assert allocator.cached_length(request) == 16 and allocator.capacity() == counts
        assert [allocator.block_table(r) for r in requests] == tables
    assert allocator.capacity() == CapacityCounts(4, 0, 4, 4, 2, 34)
    for request in requests:
        assert allocator.cached_length(request) == 17
        allocator.release_all(request)
    assert allocator.capacity() == CapacityCounts(4, 4, 0, 0, 0, 0)


@pytest.mark.parametrize("fault", ["incomplete", "order", "shape", "dtype", "device"])
def test_decode_append_rejects_incomplete_or_invalid_layer_writes(fault: str) -> None:
    # tests/unit/test_kv_cache.py:421-448
    device = cuda_device()
    allocator = KVAllocator(torch.zeros(22, 2, 2, 16, 4, 64, dtype=torch.float16, device=device))
    request = RequestId("request")
    allocator.create(KVReservation(request, 2))
    allocator.append(request, *kv_values(16, device=device))
    counts = allocator.capacity()
    key = torch.zeros(4, 64, dtype=torch.float16, device=device)
    value = key.clone()
    if fault == "shape":
        key = key[0]
    elif fault == "dtype":
        value = value.float()
    elif fault == "device":
        key = key.cpu()
    with pytest.raises(RuntimeError if fault == "incomplete" else ValueError), allocator.append_decode((request,)):
        allocator.write_decode_layer(request, 1 if fault == "order" else 0, key, value)
    assert allocator.capacity() == counts and allocator.cached_length(request) == 16
    allocator.release_all(request)
    assert allocator.capacity() == CapacityCounts(2, 2, 0, 0, 0, 0)


def test_thread_and_stream_ownership() -> None:
    # tests/unit/test_kv_cache.py:451-489, tests/gpu/test_kv_pool_cuda.py:86-94
    device = cuda_device()
    allocator = KVAllocator(torch.empty((22, 2, 2, 16, 4, 64), dtype=torch.float16, device=device))
    request = RequestId("a")
    allocator.create(KVReservation(request, 2))
    key, value = kv_values(1, device=device)
    with ThreadPoolExecutor(max_workers=1) as executor:
        for operation, args in (
            (allocator.capacity, ()),
            (allocator.append, (request, key, value)),
            (allocator.block_table, (request,)),
            (allocator.release_all, (request,)),
        ):
            with pytest.raises(RuntimeError, match="owning model worker"):
                executor.submit(operation, *args).result()
    other = torch.cuda.Stream(device=device)
    with torch.cuda.stream(other):
        for operation in (allocator.capacity, lambda: allocator.append(request, key, value),
                          lambda: allocator.read_block(request, 0)):
            with pytest.raises(RuntimeError, match="owning CUDA stream"):
                operation()
    assert allocator.cached_length(request) == 0


@pytest.mark.parametrize("fail_at", [1, 2])
def test_failed_write_launch_preserves_state_and_allows_retry(monkeypatch: pytest.MonkeyPatch, fail_at: int) -> None:
    # Host-side fault injection at the kernel boundary (the reference injects into copy_,
    # tests/unit/test_kv_cache.py:680-738): state must be unchanged and a retry must work.
    device = cuda_device()
    allocator = KVAllocator(nan_pool(4, device))
    a = RequestId("a")
    allocator.create(KVReservation(a, 4))
    allocator.append(a, *kv_values(15, device=device))
    before, table = allocator.capacity(), allocator.block_table(a)
    original = kernels_module.append_kv
    calls = 0

    def failing(*args, **kwargs):
        nonlocal calls
        calls += 1
        if calls == fail_at:
            raise RuntimeError("injected write failure")
        return original(*args, **kwargs)

    monkeypatch.setattr(kernels_module, "append_kv", failing)
    with pytest.raises(RuntimeError, match="injected write failure"):
        for _ in range(fail_at):
            allocator.append(a, *kv_values(18, start=100, device=device))
    monkeypatch.setattr(kernels_module, "append_kv", original)
    expected_length = 15 + 18 * (fail_at - 1)
    assert allocator.cached_length(a) == expected_length
    if fail_at == 1:
        assert allocator.capacity() == before and allocator.block_table(a) == table
    allocator.release_all(a)
    assert allocator.capacity() == CapacityCounts(4, 4, 0, 0, 0, 0)


def test_oracle_and_kernel_agree_on_random_prefill_positions(rope_golden: np.ndarray) -> None:
    device = cuda_device()
    allocator = KVAllocator(nan_pool(1000, device))
    oracle_pool = kv_write.new_pool(1000)
    oracle = OracleAllocator(1000, audit=False)
    generator = workloads.rng(5, 1)
    for request in range(12):
        first = int(generator.integers(1, 600))
        second = int(generator.integers(1, 600))
        credits = workloads.blocks_for(first + second)
        allocator.create(KVReservation(RequestId(str(request)), credits))
        oracle.create(request, credits)
        for tokens in (first, second):
            key = workloads.normal_f16(generator, (22, tokens, 4, 64))
            value = workloads.normal_f16(generator, (22, tokens, 4, 64))
            start = oracle.sequences[request].length
            slots = np.asarray(oracle.append(request, tokens))
            kv_write.append_rotated(oracle_pool, key, value, slots, np.arange(start, start + tokens), rope_golden)
            allocator.append(RequestId(str(request)), torch.from_numpy(key).to(device),
                             torch.from_numpy(value).to(device), rotate=True)
    allocator.check_device_errors()
    assert np.array_equal(allocator.pool.cpu().numpy().view(np.uint16), oracle_pool.view(np.uint16))
