"""The oracle pinned against golden vectors produced by the reference itself.

tests/golden/make_golden.py ran PagedCore's own kv_cache / attention / dense
code on the seeded workloads; these tests require the oracle to reproduce
those outputs bit for bit (pool bytes, tables, capacity, RoPE table) or
within the reference's own tolerance (FP32 attention, where only BLAS
summation order differs).
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from oracle import attention as oracle_attention
from oracle import kv_write, rope
from oracle.allocator import OracleAllocator
from pagedcore_b200 import workloads
from tests.conftest import SMALL_CASE


def sha256(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).view(np.uint8)).hexdigest()


def test_rope_table_matches_reference_apply_rope(rope_golden: np.ndarray) -> None:
    table = rope.cos_sin_table()
    assert table.dtype == np.float16 and table.shape == (2, 2048, 32)
    assert np.array_equal(table.view(np.uint16), rope_golden.view(np.uint16))


def test_product_rope_table_matches_reference(rope_golden: np.ndarray) -> None:
    from pagedcore_b200.rope import host_table

    assert np.array_equal(host_table().numpy().view(np.uint16), rope_golden.view(np.uint16))


def test_rope_rotation_known_answers(rope_golden: np.ndarray) -> None:
    # Position 0 is the identity (cos 1, sin 0); a unit first-half vector
    # reads back cos in the first half and sin in the second half.
    x = np.zeros((1, 1, 64), dtype=np.float16)
    x[..., :32] = 1
    out = rope.rotate(x, np.array([0]), rope_golden)
    assert np.array_equal(out, x)
    out = rope.rotate(x, np.array([1234]), rope_golden)
    assert np.array_equal(out[0, 0, :32], rope_golden[0, 1234])
    assert np.array_equal(out[0, 0, 32:], rope_golden[1, 1234])


def _build_attention_pool(case: workloads.AttentionCase) -> tuple[np.ndarray, OracleAllocator, list[int]]:
    pool = kv_write.new_pool(case.num_blocks)
    allocator = OracleAllocator(case.num_blocks, audit=False)
    allocator.free = [int(b) for b in case.free_order]
    requests = list(range(len(case.lengths)))
    for request, length, key, value in zip(requests, case.lengths, case.keys, case.values, strict=True):
        allocator.create(request, workloads.blocks_for(length))
        slots = allocator.append(request, length)
        kv_write.write_rows(pool, 0, key, value, np.asarray(slots))
    return pool, allocator, requests


def test_attention_config1_matches_reference(attention_golden: dict[str, np.ndarray]) -> None:
    case = workloads.attention_case()
    pool, allocator, requests = _build_attention_pool(case)
    tables = np.concatenate([np.asarray(allocator.table(r), dtype=np.int32) for r in requests])
    assert np.array_equal(tables, attention_golden["tables"])
    for layer in (0, 21):
        for row, request in enumerate(requests):
            out = oracle_attention.paged_attention(pool, layer, case.query[row], allocator.table(request), case.lengths[row])
            expected = attention_golden[f"out_layer{layer}"][row]
            np.testing.assert_allclose(out.astype(np.float32), expected.astype(np.float32), atol=1e-3, rtol=1e-3)
            key, value = oracle_attention.gather_dense(pool, layer, allocator.table(request), case.lengths[row])
            dense = oracle_attention.dense_fp64(case.query[row], key, value)
            assert np.array_equal(dense, attention_golden[f"dense_layer{layer}"][row])
            np.testing.assert_allclose(out.astype(np.float32), dense.astype(np.float32), atol=2e-3, rtol=2e-3)


def replay_append(case: workloads.AppendCase, table: np.ndarray) -> tuple[np.ndarray, OracleAllocator, dict]:
    pool = kv_write.new_pool(case.num_blocks)
    allocator = OracleAllocator(case.num_blocks, audit=False)
    checkpoints = {}
    for index, op in enumerate(case.churn):
        if op.kind == "create":
            allocator.create(op.request, op.credits)
            key, value = workloads.churn_fill(index, op.tokens)
            kv_write.write_rows(pool, 0, key, value, np.asarray(allocator.append(op.request, op.tokens)))
        else:
            allocator.release(op.request)
    checkpoints["after_churn"] = (allocator.capacity_unchecked(), list(allocator.free), sha256(pool))
    for prompt in case.prompts:
        allocator.create(prompt.request, prompt.credits)
        tokens = prompt.key.shape[1]
        slots = np.asarray(allocator.append(prompt.request, tokens))
        kv_write.append_rotated(pool, prompt.key, prompt.value, slots, np.arange(tokens), table)
    checkpoints["after_prompts"] = (allocator.capacity_unchecked(), sha256(pool))
    slots, positions = allocator.decode_begin(case.decode.requests)
    for layer in range(22):
        kv_write.append_rotated(
            pool, case.decode.key[layer][None], case.decode.value[layer][None], np.asarray(slots),
            np.asarray(positions), table, layer_begin=layer,
        )
    allocator.decode_commit()
    checkpoints["after_decode"] = (allocator.capacity_unchecked(), sha256(pool))
    return pool, allocator, checkpoints


def test_append_small_case_matches_reference(append_small_golden: dict, rope_golden: np.ndarray) -> None:
    case = workloads.append_case(**SMALL_CASE)
    pool, allocator, _ = replay_append(case, rope_golden)
    assert np.array_equal(pool[0].view(np.uint16), append_small_golden["pool_layer0"].view(np.uint16))
    assert np.array_equal(pool[21].view(np.uint16), append_small_golden["pool_layer21"].view(np.uint16))
    assert sha256(pool) == bytes(append_small_golden["pool_sha256"]).hex()
    assert list(allocator.capacity_unchecked()) == append_small_golden["capacity"].tolist()
    assert allocator.free == append_small_golden["free_list"].tolist()


@pytest.mark.slow
def test_append_config2_matches_reference(append_golden: dict, rope_golden: np.ndarray) -> None:
    case = workloads.append_case()
    _, allocator, checkpoints = replay_append(case, rope_golden)
    capacity, free, digest = checkpoints["after_churn"]
    assert list(capacity) == append_golden["after_churn"]["capacity"]
    assert free == append_golden["after_churn"]["free_list"]
    assert digest == append_golden["after_churn"]["pool_sha256"]
    capacity, digest = checkpoints["after_prompts"]
    assert list(capacity) == append_golden["after_prompts"]["capacity"]
    assert digest == append_golden["after_prompts"]["pool_sha256"]
    capacity, digest = checkpoints["after_decode"]
    assert list(capacity) == append_golden["after_decode"]["capacity"]
    assert digest == append_golden["after_decode"]["pool_sha256"]
    for request, table in append_golden["after_decode"]["tables"].items():
        assert list(allocator.table(int(request))) == table
        assert allocator.length(int(request)) == append_golden["after_decode"]["lengths"][request]


def test_oracle_audit_detects_corruption() -> None:
    allocator = OracleAllocator(4)
    allocator.create("a", 3)
    allocator.create("b", 1)
    allocator.append("a", 17)
    allocator.append("b", 1)
    allocator.sequences["a"].blocks = [allocator.sequences["b"].blocks[0], allocator.sequences["a"].blocks[1]]
    with pytest.raises(RuntimeError, match="KV"):
        allocator.audit()
