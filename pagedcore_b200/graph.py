"""A staged decode step of the KV path replayed as a CUDA graph.

The 22 fused decode-layer launches of a step (split kernel + combine each)
cost about 37 us of Python and ctypes per layer on the host, close to the
43 us a layer takes on the GPU.  A ``DecodeStepGraph`` captures them once
and replays them as one graph per step, so the host only stages the step
(ledger, tables, one upload) and launches the graph.

A replay repeats its launches' arguments, so nothing in them may depend on
the step's batch.  The step is staged with a fixed layout
(``append_decode(layout=(rows, pieces))``): its tables are padded to the
graph's row capacity and to one piece per resident CTA slot, so the table
addresses, the split grid (every slot; empty pieces exit at once) and the
combine grid (every row; rows without pieces exit at once) are the same
for every batch of up to ``rows`` requests.  The block count changes every
step; with piece tables the kernels use it only as a memory bound, so the
graph is given the room of the flat list in its upload buffer.  What stays
fixed is the pool, the workspace, the upload buffer (the upload alternates
between two, so a graph is kept per buffer) and the caller's
query/key/value/output buffers (a graph is kept per buffer set).  The
ledger records the 22 layers after each replay is enqueued.
"""

from __future__ import annotations

import contextlib
import gc
from collections.abc import Iterator, Sequence

import torch
from torch import Tensor

from pagedcore_b200 import kernels
from pagedcore_b200._lib import DECODE_EARLY_KV, check, lib
from pagedcore_b200.engine_types import RequestId
from pagedcore_b200.kv_cache import KVAllocator

_LAYERS = 22


@contextlib.contextmanager
def _capturing(graph: torch.cuda.CUDAGraph, stream: torch.cuda.Stream) -> Iterator[None]:
    """Capture into ``graph`` on ``stream`` with the cycle collector held off.

    A CUDA graph that its last user left in a reference cycle is destroyed
    whenever the collector runs; if that happens mid-capture, the destroy
    is a call CUDA forbids while this thread captures, and the capture is
    lost.  So dead cycles are collected first and the collector waits until
    the capture has ended.  The capture is thread-local: another thread's
    CUDA queries (a communication library's watchdog, say) cannot spoil it.
    """
    gc.collect()
    enabled = gc.isenabled()
    gc.disable()
    try:
        with torch.cuda.graph(graph, stream=stream, capture_error_mode="thread_local"):
            yield
    finally:
        if enabled:
            gc.enable()


def _replay_args(allocator: KVAllocator, rows: int, grid: int) -> tuple:
    """Fixed pkv_decode_layer arguments of the staged (padded) step, minus layer, I/O and stream.

    With piece tables the kernels take the block count only as a bound and
    ignore the arithmetic partition, so the upload's room and constants stand
    in for them: the arguments repeat from step to step and key the graphs.
    """
    staged = allocator._staged
    fixed = allocator._decode_layer_args(staged.staged_batch, rows, grid)
    return (*fixed[:8], staged.flat_capacity, grid, 1, grid, 1, *fixed[13:16])


class DecodeStepGraph:
    """Decode steps of up to ``rows`` requests through captured CUDA graphs.

    ``step(query, key, value, out, request_ids)`` does what ``append_decode``
    plus ``decode_layer`` for layers 0..21 do for ``request_ids`` (default:
    the ids given at construction), with query [22, rows, 32, 64] and
    key/value [22, rows, 4, 64] unrotated FP16 and out [22, rows, 32, 64]
    FP16; row i of each belongs to the step's i-th request, and rows past the
    batch are neither read nor written.  ``rows`` defaults to the number of
    ids given at construction.  Graphs are captured on a side stream and
    replayed on the allocator's stream.
    """

    def __init__(
        self,
        allocator: KVAllocator,
        request_ids: Sequence[RequestId] = (),
        *,
        rows: int | None = None,
        max_graphs: int = 8,
    ) -> None:
        self.allocator = allocator
        self.requests = tuple(request_ids)
        self.rows = len(self.requests) if rows is None else rows
        if self.rows < 1 or len(self.requests) > self.rows:
            raise ValueError("a decode step graph needs 1 <= len(request_ids) <= rows")
        self.grid = kernels.decode_slots(allocator.pool.device)
        self.max_graphs = max_graphs
        self._graphs: dict[tuple, torch.cuda.CUDAGraph] = {}
        self.captures = 0

    def _check(self, query: Tensor, key: Tensor, value: Tensor, out: Tensor) -> None:
        device = self.allocator.pool.device
        for name, tensor, heads in (("query", query, 32), ("key", key, 4), ("value", value, 4), ("out", out, 32)):
            if (
                tensor.shape != (_LAYERS, self.rows, heads, 64)
                or tensor.dtype != torch.float16
                or tensor.device != device
                or not tensor.is_contiguous()
            ):
                raise ValueError(f"{name} must be contiguous FP16 [22, {self.rows}, {heads}, 64] on the pool device")

    def _capture(self, args: tuple, query: Tensor, key: Tensor, value: Tensor, out: Tensor) -> torch.cuda.CUDAGraph:
        allocator = self.allocator
        (pool, num_blocks, rope, lengths, prefix, flat, pieces, row_pieces, bound, grid, per_cta, big, tail, ws,
         ws_bytes, err) = args
        side = torch.cuda.Stream(allocator.pool.device)
        side.wait_stream(allocator._stream)
        graph = torch.cuda.CUDAGraph()
        with _capturing(graph, side):
            for layer in range(_LAYERS):
                q, k, v, o = query[layer], key[layer], value[layer], out[layer]
                check(
                    lib.pkv_decode_layer(
                        pool, num_blocks, layer, q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), k.stride(0),
                        rope, lengths, prefix, flat, pieces, row_pieces, self.rows, bound, grid, per_cta, big, tail,
                        # Layers after the first follow this graph's own combine, which
                        # writes no pool data: they may start streaming early.
                        o.data_ptr(), o.stride(0), ws, ws_bytes, err, DECODE_EARLY_KV if layer else 0,
                        side.cuda_stream,
                    )
                )
        allocator._stream.wait_stream(side)
        self.captures += 1
        return graph

    @torch.inference_mode()
    def step(
        self, query: Tensor, key: Tensor, value: Tensor, out: Tensor,
        request_ids: Sequence[RequestId] | None = None,
    ) -> Tensor:
        allocator = self.allocator
        requests = self.requests if request_ids is None else tuple(request_ids)
        if not 1 <= len(requests) <= self.rows:
            raise ValueError(f"a decode step graph serves 1 to {self.rows} requests, not {len(requests)}")
        self._check(query, key, value, out)
        with allocator.append_decode(requests, layout=(self.rows, self.grid)):
            staged = allocator._staged
            args = _replay_args(allocator, self.rows, self.grid)
            cache_key = (args, query.data_ptr(), key.data_ptr(), value.data_ptr(), out.data_ptr())
            graph = self._graphs.get(cache_key)
            if graph is None:
                if len(self._graphs) >= self.max_graphs:
                    del self._graphs[next(iter(self._graphs))]  # the oldest capture
                graph = self._graphs[cache_key] = self._capture(args, query, key, value, out)
            ledger = allocator._ledger
            ledger.decode_check(-1, 0)  # a fresh staged step: layer 0 is next
            graph.replay()
            ledger.decode_mark_layers(0, _LAYERS)
            staged.written = _LAYERS
        return out


class DecoderStepGraph:
    """``BatchedDecoder`` steps of up to ``rows`` requests replayed as CUDA graphs.

    A decoder step launches nine kernels per layer (two residual-add norms,
    the fused Q/K/V and gate/up GEMMs, the decode layer's split and combine,
    the output and down projections, the SwiGLU product) plus the embedding,
    the final norm and the logits: about 200 launches whose Python and launch
    costs exceed the GPU time at small batches.  Here the whole step,
    ``BatchedDecoder.forward`` with the fused decode layer launched on the
    step's padded tables, is captured once per
    upload buffer and replayed: the host stages the step (ledger, tables, one
    upload), copies the token ids into a fixed buffer and launches the graph.
    ``step(input_ids, request_ids)`` returns the logits [B, 1, V] of
    ``BatchedDecoder.step`` for the same inputs (the GEMMs run over all
    ``rows`` rows, so their rounding may differ in the last bits).
    """

    def __init__(self, decoder, allocator: KVAllocator, *, rows: int, max_graphs: int = 4) -> None:
        if rows < 1:
            raise ValueError("a decoder step graph needs at least one row")
        self.decoder = decoder
        self.allocator = allocator
        self.rows = rows
        device = allocator.pool.device
        self.grid = kernels.decode_slots(device)
        self.max_graphs = max_graphs
        with torch.inference_mode(False):  # fixed buffers, updated in place in any mode
            self.ids = torch.zeros((rows, 1), dtype=torch.int64, device=device)
            self.attention = torch.empty((rows, 32, 64), dtype=torch.float16, device=device)
        self._graphs: dict[tuple, tuple[torch.cuda.CUDAGraph, Tensor]] = {}
        self.captures = 0

    def _capture(self, args: tuple) -> tuple[torch.cuda.CUDAGraph, Tensor]:
        allocator = self.allocator
        (pool, num_blocks, rope, lengths, prefix, flat, pieces, row_pieces, bound, grid, per_cta, big, tail, ws,
         ws_bytes, err) = args
        side = torch.cuda.Stream(allocator.pool.device)
        side.wait_stream(allocator._stream)
        out = self.attention

        def attend(layer: int, q: Tensor, k: Tensor, v: Tensor) -> Tensor:
            # The previous kernel is a GEMM of this step, not a decode combine:
            # no early K/V (it would only save the launch, which a GEMM
            # predecessor does not overlap).
            check(
                lib.pkv_decode_layer(
                    pool, num_blocks, layer, q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), k.stride(0),
                    rope, lengths, prefix, flat, pieces, row_pieces, self.rows, bound, grid, per_cta, big, tail,
                    out.data_ptr(), out.stride(0), ws, ws_bytes, err, 0, side.cuda_stream,
                )
            )
            return out

        # One forward outside the capture first, with an attention stand-in
        # that touches no pool data: cuBLAS creates its handle and workspace
        # on first use on a stream, which must not happen while capturing.
        with torch.cuda.stream(side):
            self.decoder.forward(self.ids, lambda layer, q, k, v: out)
        graph = torch.cuda.CUDAGraph()
        with _capturing(graph, side):
            logits = self.decoder.forward(self.ids, attend)
        allocator._stream.wait_stream(side)
        self.captures += 1
        return graph, logits

    @torch.inference_mode()
    def step(self, input_ids: Tensor, request_ids: Sequence[RequestId]) -> Tensor:
        allocator = self.allocator
        requests = tuple(request_ids)
        count = len(requests)
        if not 1 <= count <= self.rows:
            raise ValueError(f"a decoder step graph serves 1 to {self.rows} requests, not {count}")
        if (
            input_ids.dtype != torch.int64
            or input_ids.shape != (count, 1)
            or input_ids.device != allocator.pool.device
        ):
            raise ValueError("input_ids must be int64 [batch, 1] matching request IDs on the pool device")
        with allocator.append_decode(requests, layout=(self.rows, self.grid)):
            staged = allocator._staged
            args = _replay_args(allocator, self.rows, self.grid)
            entry = self._graphs.get(args)
            if entry is None:
                if len(self._graphs) >= self.max_graphs:
                    del self._graphs[next(iter(self._graphs))]  # the oldest capture
                entry = self._graphs[args] = self._capture(args)
            graph, logits = entry
            self.ids[:count].copy_(input_ids)
            ledger = allocator._ledger
            ledger.decode_check(-1, 0)  # a fresh staged step: layer 0 is next
            graph.replay()
            ledger.decode_mark_layers(0, _LAYERS)
            staged.written = _LAYERS
            return logits[:count].clone()
