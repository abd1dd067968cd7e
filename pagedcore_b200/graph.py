"""A staged decode step of the KV path replayed as a CUDA graph.

The 22 fused decode-layer launches of a step (split kernel + combine each)
cost about 37 us of Python and ctypes per layer on the host, close to the
43 us a layer takes on the GPU.  A ``DecodeStepGraph`` captures them once
and replays them as one graph per step, so the host only stages the step
(ledger, tables, one upload) and launches the graph.

What a replay needs fixed is fixed: the pool, the workspace, the step
tables' device buffers (the upload alternates between two, so a graph is
kept per buffer), the caller's query/key/value/output buffers (a graph is
kept per buffer set) and the number of pieces.  The block count changes
every step; with piece tables the kernels use it only as a memory bound, so
the graph is given the room of the flat list in its upload buffer.  The
ledger records the 22 layers after each replay is enqueued.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
from torch import Tensor

from pagedcore_b200._lib import DECODE_EARLY_KV, check, lib
from pagedcore_b200.engine_types import RequestId
from pagedcore_b200.kv_cache import KVAllocator

_LAYERS = 22


class DecodeStepGraph:
    """Decode steps of a fixed batch through captured CUDA graphs.

    ``step(query, key, value, out)`` does what ``append_decode`` plus
    ``decode_layer`` for layers 0..21 do, with query [22, B, 32, 64] and
    key/value [22, B, 4, 64] unrotated FP16 and out [22, B, 32, 64] FP16
    written.  Graphs are captured on a side stream and replayed on the
    allocator's stream.
    """

    def __init__(self, allocator: KVAllocator, request_ids: Sequence[RequestId], *, max_graphs: int = 8) -> None:
        self.allocator = allocator
        self.requests = tuple(request_ids)
        self.max_graphs = max_graphs
        self._graphs: dict[tuple, torch.cuda.CUDAGraph] = {}
        self.captures = 0

    def _check(self, query: Tensor, key: Tensor, value: Tensor, out: Tensor) -> None:
        count = len(self.requests)
        device = self.allocator.pool.device
        for name, tensor, heads in (("query", query, 32), ("key", key, 4), ("value", value, 4), ("out", out, 32)):
            if (
                tensor.shape != (_LAYERS, count, heads, 64)
                or tensor.dtype != torch.float16
                or tensor.device != device
                or not tensor.is_contiguous()
            ):
                raise ValueError(f"{name} must be contiguous FP16 [22, batch, {heads}, 64] on the pool device")

    def _capture(self, args: tuple, query: Tensor, key: Tensor, value: Tensor, out: Tensor) -> torch.cuda.CUDAGraph:
        allocator = self.allocator
        (pool, num_blocks, rope, lengths, prefix, flat, pieces, row_pieces, bound, grid, per_cta, big, tail, ws,
         ws_bytes, err) = args
        count = len(self.requests)
        side = torch.cuda.Stream(allocator.pool.device)
        side.wait_stream(allocator._stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for layer in range(_LAYERS):
                q, k, v, o = query[layer], key[layer], value[layer], out[layer]
                check(
                    lib.pkv_decode_layer(
                        pool, num_blocks, layer, q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), k.stride(0),
                        rope, lengths, prefix, flat, pieces, row_pieces, count, bound, grid, per_cta, big, tail,
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
    def step(self, query: Tensor, key: Tensor, value: Tensor, out: Tensor) -> Tensor:
        allocator = self.allocator
        self._check(query, key, value, out)
        with allocator.append_decode(self.requests):
            staged = allocator._staged
            batch = staged.staged_batch
            fixed = allocator._decode_layer_args(batch, len(self.requests))
            grid = batch.plan.grid
            # With piece tables the kernels take the block count only as a
            # bound and ignore the arithmetic partition: pass the step's upload
            # room and constants, so the arguments repeat from step to step.
            args = (*fixed[:8], staged.flat_capacity, grid, 1, grid, 1, *fixed[13:16])
            cache_key = (args, query.data_ptr(), key.data_ptr(), value.data_ptr(), out.data_ptr())
            graph = self._graphs.get(cache_key)
            if graph is None:
                if len(self._graphs) >= self.max_graphs:
                    self._graphs.clear()
                graph = self._graphs[cache_key] = self._capture(args, query, key, value, out)
            ledger = allocator._ledger
            ledger.decode_check(-1, 0)  # a fresh staged step: layer 0 is next
            graph.replay()
            ledger.decode_mark_layers(0, _LAYERS)
            staged.written = _LAYERS
        return out
