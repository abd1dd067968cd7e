"""The allocation-free decode attention entry point, through the C ABI.

``pkv_decode_attention_noalloc`` serves callers that cannot give this library
device memory (their device memory belongs to another allocator, or their
plugin interface has no workspace callback): it keeps its split partials in a
fixed device array instead of a caller workspace.  It must return what
``pkv_decode_attention`` returns for the same batch, bit for bit (the same
kernels, piece tables and merge order), also on a second call that finds the
previous call's data still in that array, and match the oracle.  The file is named to
be collected last; it builds its own cache so it also runs alone.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oracle_attention
from pagedcore_b200 import _lib, kernels, workloads
from pagedcore_b200.engine_types import KVReservation, RequestId
from pagedcore_b200.kv_cache import KVAllocator
from tests.conftest import cuda_device

pytestmark = pytest.mark.gpu


def _noalloc(allocator: KVAllocator, batch, query: torch.Tensor, layer: int, out: torch.Tensor) -> int:
    return _lib.lib.pkv_decode_attention_noalloc(
        allocator.pool.data_ptr(),
        allocator.pool.shape[2],
        layer,
        query.data_ptr(),
        query.stride(0),
        batch.lengths.data_ptr(),
        batch.prefix.data_ptr(),
        batch.flat.data_ptr(),
        batch.pieces.data_ptr(),
        batch.row_pieces.data_ptr(),
        len(batch.requests),
        batch.total_blocks,
        batch.plan.grid,
        batch.plan.blocks_per_cta,
        *batch.plan.pieces(),
        out.data_ptr(),
        out.stride(0),
        allocator._error.data_ptr(),
        torch.cuda.current_stream().cuda_stream,
    )


def _cache(lengths: list[int], device: torch.device) -> tuple[KVAllocator, tuple[RequestId, ...]]:
    need = sum(workloads.blocks_for(n) for n in lengths) + 4
    pool = torch.full((22, 2, need, 16, 4, 64), torch.nan, dtype=torch.float16, device=device)
    allocator = KVAllocator(pool, validation="incremental")
    allocator.ledger.reorder_free(workloads.rng(41, 1).permutation(need).astype(np.int32))
    generator = torch.Generator(device=device).manual_seed(41)
    requests = []
    for row, length in enumerate(lengths):
        request = RequestId(f"n{row}")
        allocator.create(KVReservation(request, workloads.blocks_for(length)))
        key = torch.randn(22, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
        value = torch.randn(22, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
        allocator.append(request, key, value)
        requests.append(request)
    return allocator, tuple(requests)


def test_noalloc_entry_matches_workspace_entry_on_two_calls_in_a_row() -> None:
    device = cuda_device()
    lengths = workloads.decode_lengths(43, 64, high=2048).tolist()
    allocator, requests = _cache(lengths, device)
    generator = torch.Generator(device=device).manual_seed(43)
    for layer in (3, 17):  # the second call finds the first call's partials in the array
        batch = allocator.decode_batch(requests, layer_index=layer)
        assert batch.plan.grid > 1  # rows are split, so the partials array is used
        query = torch.randn(len(lengths), 32, 64, dtype=torch.float16, device=device, generator=generator)
        expected = torch.empty_like(query)
        kernels.decode_attention(allocator.pool, layer, query, batch.lengths, batch.prefix, batch.flat,
                                 batch.total_blocks, batch.plan, expected,
                                 allocator._workspace_for(batch.plan.workspace_bytes), allocator._error,
                                 batch.pieces, batch.row_pieces)
        actual = torch.full_like(query, float("nan"))
        assert _noalloc(allocator, batch, query, layer, actual) == _lib.PKV_OK, _lib.lib.pkv_last_error()
        torch.cuda.synchronize()
        allocator.check_device_errors()
        # Same kernels, same piece tables, same merge order: the same bits.
        assert torch.equal(actual.view(torch.int16), expected.view(torch.int16))
        # And the reference's algorithm (the oracle's FP32 page loop) on a few rows.
        layer_pool = allocator.pool[layer].cpu().numpy()[None]
        got = actual.cpu().numpy().astype(np.float32)
        q = query.cpu().numpy()
        for row in (0, int(np.argmax(lengths)), len(lengths) - 1):
            request = requests[row]
            reference = oracle_attention.paged_attention(layer_pool, 0, q[row], allocator.block_table(request),
                                                         allocator.cached_length(request))
            np.testing.assert_allclose(got[row], reference.astype(np.float32), atol=2e-3, rtol=1e-2)


def test_noalloc_entry_rejects_batches_beyond_its_fixed_array() -> None:
    # Refused on the host before any launch: the plan's workspace must fit in 8 MiB
    # (2048 + 16 * grid + 8448 * (batch + grid) bytes: 990 + 1000 rows is far over).
    cuda_device()
    status = _lib.lib.pkv_decode_attention_noalloc(
        None, 1, 0, None, 0, None, None, None, None, None, 990, 1000, 10, 100, 10, 100, None, 0, None, None
    )
    assert status == _lib.PKV_VALUE_ERROR
    assert b"over the static scratch limit of 8388608" in _lib.lib.pkv_last_error()
