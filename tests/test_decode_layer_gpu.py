"""The fused decode layer (RoPE + new-token KV write + attention + in-kernel merge).

It must leave exactly the pool the separate path leaves (append kernel with
fused RoPE, then the two-pass attention), produce bit-identical attention
(same tiles, same merge order), and match the oracle for every split plan.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oracle_attention
from oracle import kv_write, rope
from pagedcore_b200 import kernels, workloads
from pagedcore_b200.attention import paged_decode_attention
from pagedcore_b200.engine_types import KVReservation, RequestId
from pagedcore_b200.kv_cache import KVAllocator
from tests.conftest import cuda_device

pytestmark = pytest.mark.gpu


def build(lengths, seed: int, device: torch.device, copies: int = 1):
    """Identical fragmented pools/allocators holding the same prompts (room for +2 tokens)."""
    need = sum(workloads.blocks_for(n + 2) for n in lengths) + 8
    order = workloads.rng(seed, 7).permutation(need).astype(np.int32)
    generator = torch.Generator(device=device).manual_seed(seed)
    prompts = []
    for length in lengths:
        key = torch.randn(22, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
        value = torch.randn(22, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
        prompts.append((key, value))
    allocators = []
    for _ in range(copies):
        pool = torch.full((22, 2, need, 16, 4, 64), torch.nan, dtype=torch.float16, device=device)
        allocator = KVAllocator(pool, validation="incremental")
        allocator.ledger.reorder_free(order)
        for row, (key, value) in enumerate(prompts):
            request = RequestId(f"r{row}")
            allocator.create(KVReservation(request, workloads.blocks_for(lengths[row] + 2)))
            allocator.append(request, key, value, rotate=True)
        allocators.append(allocator)
    requests = tuple(RequestId(f"r{row}") for row in range(len(lengths)))
    return allocators, requests


def step_inputs(count: int, seed: int, device: torch.device):
    q, k, v = workloads.decode_step_inputs(seed, count, 0)
    return tuple(torch.from_numpy(x).to(device) for x in (q, k, v))


LENGTHS = [1, 15, 16, 17, 31, 32, 33, 100, 255, 256, 700, 2000, 1200, 64, 5]


def test_fused_layer_matches_separate_path_bit_for_bit() -> None:
    device = cuda_device()
    (fused, separate), requests = build(LENGTHS, 5, device, copies=2)
    q, k, v = step_inputs(len(LENGTHS), 5, device)
    fused_out, separate_out = [], []
    with fused.append_decode(requests):
        for layer in range(22):
            fused_out.append(fused.decode_layer(layer, q[layer], k[layer], v[layer]))
    with separate.append_decode(requests):
        for layer in range(22):
            q_rot = separate.write_decode_batch(layer, k[layer], v[layer], query=q[layer], rotate=True)
            separate_out.append(paged_decode_attention(q_rot, separate, requests, layer_index=layer))
    torch.cuda.synchronize()
    fused.check_device_errors()
    separate.check_device_errors()
    assert torch.equal(fused.pool.view(torch.int16), separate.pool.view(torch.int16))
    for layer in range(22):
        assert torch.equal(fused_out[layer], separate_out[layer]), layer
    assert fused.capacity() == separate.capacity()
    assert [fused.cached_length(r) for r in requests] == [n + 1 for n in LENGTHS]


# (blocks_per_cta, big_ctas, tail_blocks): uniform splits (big_ctas 0) and
# two-tier splits, big pieces followed by tail pieces.
@pytest.mark.parametrize("pieces", [(1, 0, 0), (2, 0, 0), (3, 0, 0), (7, 0, 0), (16, 0, 0), (300, 0, 0), (20, 10, 3),
                                    (7, 30, 1), (100, 2, 5)])
def test_fused_layer_matches_oracle_under_every_plan(pieces: tuple[int, int, int], rope_golden: np.ndarray) -> None:
    device = cuda_device()
    (allocator,), requests = build(LENGTHS, 6, device)
    count = len(LENGTHS)
    q, k, v = step_inputs(count, 6, device)
    before = allocator.pool.cpu().numpy()
    outputs = []
    with allocator.append_decode(requests):
        staged = allocator._staged
        batch = allocator._upload_batch(staged.requests, staged.handles, -2)
        plan = kernels.DecodePlan.split(count, batch.total_blocks, *pieces)
        workspace = torch.zeros(plan.workspace_bytes // 4, dtype=torch.float32, device=device)
        for layer in range(22):
            allocator.ledger.decode_check(-1, layer)
            out = torch.empty(count, 32, 64, dtype=torch.float16, device=device)
            kernels.decode_layer(allocator.pool, layer, q[layer], k[layer], v[layer], allocator._rope, batch.lengths,
                                 batch.prefix, batch.flat, batch.total_blocks, plan, out, workspace,
                                 allocator._error)
            allocator.ledger.decode_mark(-1, layer)
            outputs.append(out)
    torch.cuda.synchronize()
    allocator.check_device_errors()

    # Oracle: the same staged append on a copy of the pool, then the reference attention.
    oracle_pool = before.copy()
    positions = np.array(LENGTHS)
    slots = []
    for request, length in zip(requests, LENGTHS, strict=True):
        table = allocator.block_table(request)
        slots.append(table[length // 16] * 16 + length % 16)
    q_np, k_np, v_np = (x.cpu().numpy() for x in (q, k, v))
    for layer in range(22):
        kv_write.append_rotated(oracle_pool, k_np[layer][None], v_np[layer][None], np.asarray(slots), positions,
                                rope_golden, layer_begin=layer)
    assert np.array_equal(allocator.pool.cpu().numpy().view(np.uint16), oracle_pool.view(np.uint16))
    for layer in (0, 9, 21):
        q_rot = rope.rotate(q_np[layer][None], positions, rope_golden)[0]
        got = outputs[layer].cpu().numpy().astype(np.float32)
        for row, request in enumerate(requests):
            expected = oracle_attention.paged_attention(
                oracle_pool, layer, q_rot[row], allocator.block_table(request), LENGTHS[row] + 1
            ).astype(np.float32)
            np.testing.assert_allclose(got[row], expected, atol=2e-3, rtol=1e-2)


def test_fused_layer_validates_order_and_shapes() -> None:
    device = cuda_device()
    (allocator,), requests = build([5, 20], 8, device)
    q, k, v = step_inputs(2, 8, device)
    with pytest.raises(RuntimeError, match="staged append"):
        allocator.decode_layer(0, q[0], k[0], v[0])
    with allocator.append_decode(requests):
        with pytest.raises(ValueError, match="once in order"):
            allocator.decode_layer(1, q[1], k[1], v[1])
        with pytest.raises(ValueError, match="K and V must share"):
            allocator.decode_layer(0, q[0], k[0][:1], v[0][:1])
        with pytest.raises(ValueError, match="query must be FP16"):
            allocator.decode_layer(0, q[0].float(), k[0], v[0])
        for layer in range(22):
            allocator.decode_layer(layer, q[layer], k[layer], v[layer])
    assert [allocator.cached_length(r) for r in requests] == [6, 21]
