"""Causal prompt attention through the block table (pkv_prefill_attention).

Chunks are written with the append kernel (RoPE fused) into a fragmented,
NaN-filled pool; then every token t of a chunk starting at position `start`
must attend to positions 0 .. start + t exactly as the oracle's paged
attention does for a row of that length (the reference's FP32 algorithm,
attention.py:32-53), and as the split-K decode kernel does when it serves each
token as a row, up to the full 2048-position context.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oracle_attention
from pagedcore_b200 import kernels, workloads
from pagedcore_b200.engine_types import KVReservation, RequestId
from pagedcore_b200.kv_cache import KVAllocator
from tests.conftest import cuda_device

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2  # FP32 accumulation, one FP16 rounding: the decode attention's bound


def fragmented_allocator(blocks: int, seed: int, device: torch.device) -> KVAllocator:
    need = blocks + 8
    pool = torch.full((22, 2, need, 16, 4, 64), torch.nan, dtype=torch.float16, device=device)
    allocator = KVAllocator(pool, validation="incremental")
    allocator.ledger.reorder_free(workloads.rng(seed, 11).permutation(need).astype(np.int32))
    return allocator


def chunk_inputs(tokens: int, seed: int, device: torch.device):
    generator = torch.Generator(device=device).manual_seed(seed)
    query = torch.randn(tokens, 32, 64, dtype=torch.float16, device=device, generator=generator)
    key = torch.randn(tokens, 4, 64, dtype=torch.float16, device=device, generator=generator)
    value = torch.randn(tokens, 4, 64, dtype=torch.float16, device=device, generator=generator)
    return query, key, value


def prefill_chunks(allocator: KVAllocator, request: RequestId, chunks, layers, seed: int, check) -> None:
    """Prefill `chunks` tokens one chunk after another, calling check(chunk, layer, rotated, got)."""
    for index, tokens in enumerate(chunks):
        query, key, value = chunk_inputs(tokens, seed + index, allocator.pool.device)
        with allocator.prefill_append(request, tokens) as chunk:
            for layer in layers:
                rotated = chunk.write_layer(layer, key, value, query)
                check(chunk, layer, rotated, chunk.attend(layer, rotated))


@pytest.mark.parametrize(
    "chunks",
    [(1,), (15,), (16,), (17,), (49,), (130,), (20, 29), (5, 1, 40), (16, 16, 3), (33, 64)],
)
def test_prefill_attention_matches_the_oracle_for_every_token(chunks) -> None:
    device = cuda_device()
    total = sum(chunks)
    allocator = fragmented_allocator(-(-total // 16), 3, device)
    request = RequestId("p")
    allocator.create(KVReservation(request, -(-total // 16)))

    def check(chunk, layer, rotated, got):
        pool = allocator.pool.cpu().numpy()
        blocks = chunk.blocks.cpu().numpy().tolist()
        q = rotated.cpu().numpy()
        out = got.cpu().numpy().astype(np.float32)
        for t in range(chunk.tokens):
            length = chunk.start + t + 1
            expected = oracle_attention.paged_attention(pool, layer, q[t], blocks[: -(-length // 16)], length)
            np.testing.assert_allclose(out[t], expected.astype(np.float32), atol=ATOL, rtol=RTOL)
        split = chunk.attend_split(layer, rotated)
        torch.testing.assert_close(got, split, atol=ATOL, rtol=RTOL)

    prefill_chunks(allocator, request, chunks, (0, 21), 7, check)
    assert allocator.cached_length(request) == total
    allocator.check_device_errors()


# (300, 1200): a long chunk that continues a cache (start 300 shifts the
# diagonal block and every tile's block count); at these lengths each
# persistent CTA walks more than one (tile, head) item.  (2000, 47): a short
# chunk at the end of a full cache, few items that each walk every block.
@pytest.mark.parametrize("chunks", [(2047,), (1000, 1048), (300, 1200), (2000, 47)])
def test_prefill_attention_at_the_full_context(chunks) -> None:
    device = cuda_device()
    allocator = fragmented_allocator(128, 5, device)
    request = RequestId("long")
    allocator.create(KVReservation(request, 128))

    def check(chunk, layer, rotated, got):
        split = chunk.attend_split(layer, rotated)
        torch.testing.assert_close(got, split, atol=ATOL, rtol=RTOL)
        assert torch.isfinite(got).all()
        pool = allocator.pool.cpu().numpy()
        blocks = chunk.blocks.cpu().numpy().tolist()
        q = rotated.cpu().numpy()
        out = got.cpu().numpy().astype(np.float32)
        for t in sorted({0, 1, 15, 16, 17, chunk.tokens // 2, chunk.tokens - 2, chunk.tokens - 1}):
            length = chunk.start + t + 1
            expected = oracle_attention.paged_attention(pool, layer, q[t], blocks[: -(-length // 16)], length)
            np.testing.assert_allclose(out[t], expected.astype(np.float32), atol=ATOL, rtol=RTOL)

    prefill_chunks(allocator, request, chunks, (9,), 11, check)
    assert allocator.cached_length(request) == sum(chunks)
    allocator.check_device_errors()


def test_prefill_attention_checks_its_arguments_and_flags_bad_blocks() -> None:
    device = cuda_device()
    allocator = fragmented_allocator(4, 1, device)
    pool = allocator.pool
    query, _, _ = chunk_inputs(20, 2, device)
    out = torch.empty_like(query)
    flag = torch.zeros(1, dtype=torch.int32, device=device)
    blocks = torch.tensor([0, 1], dtype=torch.int32, device=device)
    with pytest.raises(ValueError, match="22 decoder layers"):
        kernels.prefill_attention(pool, 22, query, blocks, 0, out, flag)
    with pytest.raises(ValueError, match="one entry per 16 positions"):
        kernels.prefill_attention(pool, 0, query, blocks[:1], 0, out, flag)
    with pytest.raises(ValueError, match="positions below 2048"):
        many = torch.zeros(129, dtype=torch.int32, device=device)
        kernels.prefill_attention(pool, 0, query, many, 2040, out, flag)
    # A block id outside the pool reads as zeros and sets the device flag.
    pool[0, :, :2].zero_()
    bad = torch.tensor([0, pool.shape[2]], dtype=torch.int32, device=device)
    kernels.prefill_attention(pool, 0, query, bad, 0, out, flag)
    assert int(flag.item()) == 1  # PKV_DEVICE_BAD_BLOCK
    assert torch.isfinite(out).all()


def test_in_place_query_rotation_matches_the_copying_one() -> None:
    # BatchedDecoder.prefill rotates Q inside the fused Q/K/V projection output
    # (token stride 2560); it must equal the rotation into a fresh buffer.
    device = cuda_device()
    allocator = fragmented_allocator(8, 4, device)
    request = RequestId("q")
    allocator.create(KVReservation(request, 8))
    tokens = 100
    generator = torch.Generator(device=device).manual_seed(9)
    qkv = torch.randn(tokens, 2560, dtype=torch.float16, device=device, generator=generator)
    query = qkv[:, :2048].view(tokens, 32, 64)
    key = qkv[:, 2048:2304].view(tokens, 4, 64)
    value = qkv[:, 2304:].view(tokens, 4, 64)
    with allocator.prefill_append(request, tokens) as chunk:
        copied = chunk.write_layer(2, key, value, query.clone())
        rotated = chunk.write_layer(2, key, value, query, in_place=True)
        assert rotated.data_ptr() == qkv.data_ptr() and rotated.stride() == (2560, 64, 1)
        assert torch.equal(rotated, copied)
        torch.testing.assert_close(chunk.attend(2, rotated), chunk.attend(2, copied), atol=0.0, rtol=0.0)
    allocator.check_device_errors()
