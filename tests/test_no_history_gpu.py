"""No decode path materialises KV history in device memory.

The reference guards its paged decode with a dispatch mode that fails any op
producing more than one 16 x 4 x 64 page of KV (tests/conftest.py:45-85).
Here the kernels read pages straight from the pool into shared memory, so the
equivalent is an allocation bound.  After warm-up (persistent workspace and
table buffers exist), a staged decode step through the fused per-layer path
or through ``DecodeStepGraph`` allocates at most one page on the device
(nothing, in practice), and the two-pass path allocates only its int32 block
tables, never KV-sized data, while it streams hundreds of MB of K/V.
"""

from __future__ import annotations

import pytest
import torch

from pagedcore_b200 import workloads
from pagedcore_b200.attention import paged_decode_attention
from pagedcore_b200.engine_types import KVReservation, RequestId
from pagedcore_b200.graph import DecodeStepGraph
from pagedcore_b200.kv_cache import KVAllocator
from tests.conftest import cuda_device

pytestmark = pytest.mark.gpu

PAGE_BYTES = 16 * 4 * 64 * 2  # one block of one layer's K (or V)


@pytest.fixture(scope="module")
def batch():
    device = cuda_device()
    lengths = workloads.decode_lengths(17, 64, high=1900).tolist()
    need = sum(-(-(n + 16) // 16) for n in lengths) + 4
    pool = torch.empty((22, 2, need, 16, 4, 64), dtype=torch.float16, device=device)
    allocator = KVAllocator(pool, validation="incremental")
    requests = tuple(RequestId(f"h{i}") for i in range(len(lengths)))
    generator = torch.Generator(device=device).manual_seed(17)
    for request, length in zip(requests, lengths, strict=True):
        allocator.create(KVReservation(request, -(-(length + 16) // 16)))
        kv = torch.randn(22, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
        allocator.append(request, kv, kv, rotate=True)
    rows = len(requests)
    q = torch.randn(22, rows, 32, 64, dtype=torch.float16, device=device, generator=generator)
    k = torch.randn(22, rows, 4, 64, dtype=torch.float16, device=device, generator=generator)
    out = torch.empty(22, rows, 32, 64, dtype=torch.float16, device=device)
    return allocator, requests, q, k, out, sum(lengths) * 22 * 1024


def peak_during(fn) -> int:
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    fn()
    torch.cuda.synchronize()
    return torch.cuda.max_memory_allocated() - before


def test_fused_and_graph_decode_steps_allocate_no_kv(batch) -> None:
    allocator, requests, q, k, out, kv_bytes = batch

    def fused_step() -> None:
        with allocator.append_decode(requests):
            for layer in range(22):
                allocator.decode_layer(layer, q[layer], k[layer], k[layer], out=out[layer])

    engine = DecodeStepGraph(allocator, requests)
    for _ in range(3):  # workspace, upload ring and graphs exist afterwards
        fused_step()
        engine.step(q, k, k, out)
    assert kv_bytes > 100 * 2**20
    assert peak_during(fused_step) <= PAGE_BYTES
    assert peak_during(lambda: engine.step(q, k, k, out)) <= PAGE_BYTES
    allocator.check_device_errors()


def test_two_pass_attention_allocates_only_its_tables(batch) -> None:
    allocator, requests, q, _, out, kv_bytes = batch
    rows = len(requests)
    blocks = sum(len(allocator.block_table(r)) for r in requests)
    for _ in range(2):
        paged_decode_attention(q[0], allocator, requests, layer_index=3, out=out[0])
    peak = peak_during(lambda: paged_decode_attention(q[0], allocator, requests, layer_index=3, out=out[0]))
    # pieces, row pieces, lengths, prefix and the flat table, int32, in the caching allocator's 512 B granules
    table_bytes = 4 * (4 * 444 + 4 * rows + 1 + blocks)
    assert peak <= table_bytes + 2 * 512
    assert peak < kv_bytes // 22 // 1000  # against the tens of MB streamed per layer
    allocator.check_device_errors()
