"""Per-SM slot claims of the decode kernel under uneven CTA placement.

When a decode launch is one full wave of CTAs, each CTA takes its piece by the
SM it runs on (slot s * 3 + j for the j-th CTA on SM s), and a CTA that finds
its SM's slots taken takes a free slot of another SM.  On an idle GPU every SM
receives exactly three CTAs, so the second path only runs when the placement
is uneven.  Here a long decode launch on one stream holds every slot while a
short full-wave launch (about one block per piece) on a second allocator and
stream fills slots as they free: SMs that free early receive a fourth, fifth,
... CTA of the short launch.  Which SM runs a piece changes nothing in the
arithmetic (pieces and merge order are fixed by the tables), so both launches
must reproduce their idle results bit for bit, and no kernel may flag an error.
"""

from __future__ import annotations

import pytest
import torch

from pagedcore_b200 import kernels, workloads
from pagedcore_b200.engine_types import KVReservation, RequestId
from pagedcore_b200.kv_cache import KVAllocator
from tests.conftest import cuda_device

pytestmark = pytest.mark.gpu


def filled_allocator(lengths, seed, device, stream):
    need = sum(-(-n // 16) for n in lengths) + 4
    requests = tuple(RequestId(f"c{seed}_{i}") for i in range(len(lengths)))
    with torch.cuda.stream(stream):
        pool = torch.full((22, 2, need, 16, 4, 64), torch.nan, dtype=torch.float16, device=device)
        allocator = KVAllocator(pool, validation="incremental")
        generator = torch.Generator(device=device).manual_seed(seed)
        for request, length in zip(requests, lengths, strict=True):
            allocator.create(KVReservation(request, -(-length // 16)))
            kv = torch.randn(22, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
            allocator.append(request, kv, kv * 0.5)
        query = torch.randn(len(lengths), 32, 64, dtype=torch.float16, device=device, generator=generator)
    return allocator, requests, query


def attend_layers(allocator, requests, query, stream, layers):
    with torch.cuda.stream(stream):
        batch = allocator.decode_batch(requests, layer_index=0)
        return [allocator.attend(batch, query, layer_index=layer) for layer in layers]


def test_claims_stay_exact_when_ctas_land_unevenly() -> None:
    device = cuda_device()
    slots = kernels.decode_slots(device)
    long_stream, short_stream = torch.cuda.Stream(device), torch.cuda.Stream(device)
    # Long: ~16k blocks, ~40 us per launch.  Short: just over one block per slot.
    long_alloc, long_requests, long_query = filled_allocator(
        workloads.decode_lengths(41, 256, high=1990).tolist(), 41, device, long_stream)
    short_lengths = [16] * (slots + 8)  # one block per row: slots + 8 blocks, a full wave
    short_alloc, short_requests, short_query = filled_allocator(short_lengths, 42, device, short_stream)
    with torch.cuda.stream(short_stream):  # a full wave: its CTAs claim slots by SM
        assert short_alloc.decode_batch(short_requests, layer_index=0).plan.grid == slots
    torch.cuda.synchronize()
    layers = list(range(22))

    # Idle references, one launch at a time.
    long_idle = attend_layers(long_alloc, long_requests, long_query, long_stream, layers)
    torch.cuda.synchronize()
    short_idle = attend_layers(short_alloc, short_requests, short_query, short_stream, layers)
    torch.cuda.synchronize()

    # Concurrent: the short launches queue behind the long ones' CTAs.
    for _ in range(3):
        long_busy = attend_layers(long_alloc, long_requests, long_query, long_stream, layers)
        short_busy = attend_layers(short_alloc, short_requests, short_query, short_stream, layers)
        torch.cuda.synchronize()
        for idle, busy in zip(long_idle + short_idle, long_busy + short_busy, strict=True):
            assert torch.equal(idle, busy)
    with torch.cuda.stream(long_stream):
        long_alloc.check_device_errors()
    with torch.cuda.stream(short_stream):
        short_alloc.check_device_errors()
