"""A staged decode step replayed as a CUDA graph (pagedcore_b200.graph).

The graph launches exactly the kernels ``decode_layer`` launches, with the
same tables, so outputs and pool bytes match the per-layer path bit for bit,
over steps that alternate the upload buffers and the caller's buffer sets.
"""

from __future__ import annotations

import gc

import numpy as np
import pytest
import torch

from pagedcore_b200 import workloads
from pagedcore_b200.engine_types import KVReservation, RequestId
from pagedcore_b200.graph import DecodeStepGraph, _capturing
from pagedcore_b200.kv_cache import KVAllocator
from tests.conftest import cuda_device

pytestmark = pytest.mark.gpu


def twin_allocators(lengths, device):
    need = sum(-(-(n + 12) // 16) for n in lengths) + 4
    requests = tuple(RequestId(f"g{i}") for i in range(len(lengths)))
    out = []
    for _ in range(2):
        pool = torch.full((22, 2, need, 16, 4, 64), torch.nan, dtype=torch.float16, device=device)
        allocator = KVAllocator(pool, validation="incremental")
        generator = torch.Generator(device=device).manual_seed(21)
        for request, length in zip(requests, lengths, strict=True):
            allocator.create(KVReservation(request, -(-(length + 12) // 16)))
            kv = torch.randn(22, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
            allocator.append(request, kv, kv * 0.5)
        out.append(allocator)
    return out, requests


def test_graph_steps_match_per_layer_launches_bit_for_bit() -> None:
    device = cuda_device()
    lengths = workloads.decode_lengths(21, 40, high=1500).tolist()
    (graphed, plain), requests = twin_allocators(lengths, device)
    count = len(lengths)
    generator = torch.Generator(device=device).manual_seed(22)
    sets = [
        tuple(torch.randn(22, count, h, 64, dtype=torch.float16, device=device, generator=generator) for h in (32, 4, 4))
        for _ in range(2)
    ]
    outs = [torch.empty(22, count, 32, 64, dtype=torch.float16, device=device) for _ in range(2)]
    engine = DecodeStepGraph(graphed, requests)
    for step in range(6):
        which = (step // 2) % 2  # with the alternating upload buffers: all four pairs
        q, k, v = sets[which]
        out_graph = outs[which]
        out_graph.fill_(float("nan"))
        engine.step(q, k, v, out_graph)
        out_plain = torch.empty_like(out_graph)
        with plain.append_decode(requests):
            for layer in range(22):
                plain.decode_layer(layer, q[layer], k[layer], v[layer], out=out_plain[layer])
        torch.cuda.synchronize()
        assert torch.equal(out_graph, out_plain), step
    assert engine.captures == 4  # two upload buffers x two caller buffer sets
    assert torch.equal(graphed.pool.view(torch.int16), plain.pool.view(torch.int16))
    assert [graphed.cached_length(r) for r in requests] == [n + 6 for n in lengths]
    assert graphed.capacity() == plain.capacity()
    graphed.check_device_errors()
    plain.check_device_errors()


def test_one_graph_serves_batches_of_every_size_and_order() -> None:
    device = cuda_device()
    lengths = workloads.decode_lengths(23, 40, high=1500).tolist()
    (graphed, plain), requests = twin_allocators(lengths, device)
    rows = len(requests)
    generator = torch.Generator(device=device).manual_seed(24)
    q, k, v = (torch.randn(22, rows, h, 64, dtype=torch.float16, device=device, generator=generator) for h in (32, 4, 4))
    out_graph = torch.empty(22, rows, 32, 64, dtype=torch.float16, device=device)
    engine = DecodeStepGraph(graphed, rows=rows)
    order = np.random.default_rng(25)
    for step, count in enumerate((rows, 1, 17, 33, 2, rows, 9, 40)):
        chosen = tuple(requests[i] for i in order.permutation(rows)[:count])
        out_graph.fill_(float("nan"))
        engine.step(q, k, v, out_graph, chosen)
        out_plain = torch.empty(22, count, 32, 64, dtype=torch.float16, device=device)
        with plain.append_decode(chosen):
            for layer in range(22):
                plain.decode_layer(layer, q[layer, :count], k[layer, :count], v[layer, :count], out=out_plain[layer])
        torch.cuda.synchronize()
        assert torch.equal(out_graph[:, :count], out_plain), step
        assert torch.isnan(out_graph[:, count:]).all(), step  # rows past the batch are not written
    assert engine.captures == 2  # one per upload buffer, whatever the batch
    assert torch.equal(graphed.pool.view(torch.int16), plain.pool.view(torch.int16))
    assert [graphed.cached_length(r) for r in requests] == [plain.cached_length(r) for r in requests]
    assert graphed.capacity() == plain.capacity()
    with pytest.raises(ValueError, match="serves 1 to 40"):
        engine.step(q, k, v, out_graph, requests + requests[:1])
    assert graphed.capacity() == plain.capacity()
    graphed.check_device_errors()
    plain.check_device_errors()


def test_graph_step_rejects_buffers_of_the_wrong_shape() -> None:
    device = cuda_device()
    (allocator, _), requests = twin_allocators([5, 30], device)
    engine = DecodeStepGraph(allocator, requests)
    q = torch.zeros(22, 2, 32, 64, dtype=torch.float16, device=device)
    kv = torch.zeros(22, 2, 4, 64, dtype=torch.float16, device=device)
    with pytest.raises(ValueError, match="key must be"):
        engine.step(q, kv[:, :1], kv, torch.empty_like(q))
    assert [allocator.cached_length(r) for r in requests] == [5, 30]


def test_a_graph_dropped_in_a_reference_cycle_mid_capture_does_not_spoil_it() -> None:
    """A CUDA graph left in a reference cycle is destroyed when the cycle
    collector runs.  Dropped during a capture, with a collection due at every
    allocation, it must wait: destroying it mid-capture would lose the
    capture.  The capture then replays, and the old graph is freed once the
    capture has ended."""
    device = cuda_device()
    x = torch.ones(4, device=device)
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    old = torch.cuda.CUDAGraph()
    with _capturing(old, side):
        x.add_(1)
    threshold = gc.get_threshold()
    graph = torch.cuda.CUDAGraph()
    try:
        gc.set_threshold(1, 1, 1)
        with _capturing(graph, side):
            x.mul_(3)
            cycle = [old]
            cycle.append(cycle)
            del old, cycle
            kept = [[] for _ in range(1000)]  # each list kept makes a collection due
            del kept
    finally:
        gc.set_threshold(*threshold)
    torch.cuda.current_stream(device).wait_stream(side)
    graph.replay()  # captured work is not run at capture: x goes from 1 to 3
    torch.cuda.synchronize(device)
    assert x.tolist() == [3.0] * 4
    gc.collect()  # the old graph, never replayed, is freed outside any capture
