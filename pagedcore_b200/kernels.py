"""Torch-tensor wrappers of the device entry points of ``libpagedkv.so``.

These functions only check tensor properties and pass raw pointers, sizes and
the current CUDA stream across the C ABI; all device work is done by the
sm_100a kernels in ``csrc/``.  Every function raises if the library is
missing or a tensor is not on a CUDA device: there is no non-native path.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np
import torch
from torch import Tensor

from pagedcore_b200._lib import check, lib

_LAYERS = 22
_KV_HEADS = 4
_QUERY_HEADS = 32
_HEAD_DIM = 64
_PARTIAL_BYTES = _QUERY_HEADS * (_HEAD_DIM + 2) * 4  # one split partial: (m, l, O) of 32 heads, FP32
CLAIM_BYTES = 2 * 256 * 4  # the workspace's two sets of 256 per-SM slot-claim counters (int32)


def workspace_bytes(batch: int, grid: int) -> int:
    """Workspace of a plan: 2 x 256 int32 slot-claim counters (the first 2 KiB),
    four uint32 wall-time counters per slot, then a split partial per (row,
    piece) slot (batch + grid).  It must be zero before its first use; the
    kernels leave the claim counters at zero."""
    return CLAIM_BYTES + grid * 16 + (batch + grid) * _PARTIAL_BYTES


def _ptr(tensor: Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if tensor is None else tensor.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(name: str, tensor: Tensor, device: torch.device) -> None:
    if tensor.device != device or tensor.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor on {device}")


def _kv_rows_ok(tensor: Tensor) -> bool:
    """Inner [4, 64] contiguous and 16-byte aligned rows, as the kernel reads them."""
    return (
        tensor.stride(2) == _HEAD_DIM
        and tensor.stride(3) == 1
        and tensor.stride(0) % 8 == 0
        and tensor.stride(1) % 8 == 0
        and tensor.data_ptr() % 16 == 0
    )


def append_kv(
    pool: Tensor,
    key: Tensor,
    value: Tensor,
    slots: Tensor,
    *,
    layer_begin: int,
    error_flag: Tensor,
    positions: Tensor | None = None,
    rope_table: Tensor | None = None,
    query_in: Tensor | None = None,
    query_out: Tensor | None = None,
) -> None:
    """Scatter FP16 K/V [layers, tokens, 4, 64] into the pool at ``slots``.

    With ``rope_table`` the K rows (and ``query_in`` [layers, tokens, 32, 64],
    written rotated to ``query_out``) are rotated at ``positions`` first.
    """
    device = pool.device
    for name, tensor in (("key", key), ("value", value), ("slots", slots), ("error_flag", error_flag)):
        _require_cuda(name, tensor, device)
    if key.ndim != 4 or key.shape[2:] != (_KV_HEADS, _HEAD_DIM) or value.shape != key.shape:
        raise ValueError("K and V must share FP16 [layers, tokens, 4, 64]")
    if key.dtype != torch.float16 or value.dtype != torch.float16:
        raise ValueError("K and V must be FP16")
    if not (_kv_rows_ok(key) and value.stride() == key.stride()):
        key, value = key.contiguous(), value.contiguous()
    layers, tokens = key.shape[0], key.shape[1]
    if slots.dtype != torch.int32 or slots.numel() < tokens:
        raise ValueError("slots must be int32 with one entry per token")
    if query_in is not None:
        if query_out is None or query_in.shape != (layers, tokens, _QUERY_HEADS, _HEAD_DIM):
            raise ValueError("query must be FP16 [layers, tokens, 32, 64] with an output buffer")
        # In place (query_out is query_in): the kernel reads each 16-byte chunk
        # once before writing it, through the same strides.
        in_place = (
            query_out.data_ptr() == query_in.data_ptr()
            and query_out.stride() == query_in.stride()
            and query_out.shape == query_in.shape
        )
        if not (in_place and query_in.stride()[2:] == (_HEAD_DIM, 1)):
            query_in = query_in.contiguous()
            if query_out.shape != query_in.shape or not query_out.is_contiguous():
                raise ValueError("query_out must be a contiguous buffer shaped like query, or query itself")
    check(
        lib.pkv_append_kv(
            _ptr(pool),
            pool.shape[2],
            layer_begin,
            layers,
            _ptr(key),
            _ptr(value),
            key.stride(0),
            key.stride(1),
            _ptr(slots),
            _ptr(positions),
            tokens,
            _ptr(rope_table),
            _ptr(query_in),
            _ptr(query_out),
            0 if query_in is None else query_in.stride(0),
            0 if query_in is None else query_in.stride(1),
            _ptr(error_flag),
            _stream(device),
        )
    )


@dataclass(frozen=True, slots=True)
class DecodePlan:
    """Split of a batch's flat block list into one contiguous piece per CTA.

    ``big_ctas`` pieces of ``blocks_per_cta`` blocks come first, then
    ``grid - big_ctas`` pieces of ``tail_blocks`` blocks; ``big_ctas == 0``
    stands for the uniform split (every piece ``blocks_per_cta`` blocks).
    """

    grid: int
    blocks_per_cta: int
    workspace_bytes: int
    big_ctas: int = 0
    tail_blocks: int = 0

    @classmethod
    def split(cls, batch: int, total_blocks: int, blocks_per_cta: int, big_ctas: int = 0,
              tail_blocks: int = 0) -> DecodePlan:
        """A plan with the given piece sizes (pkv_decode_plan picks its own)."""
        if big_ctas == 0:
            grid = -(-total_blocks // blocks_per_cta)
        else:
            grid = big_ctas + -(-(total_blocks - big_ctas * blocks_per_cta) // tail_blocks)
        return cls(grid, blocks_per_cta, workspace_bytes(batch, grid), big_ctas, tail_blocks)

    def pieces(self) -> tuple[int, int]:
        """(big_ctas, tail_blocks) as the C ABI takes them."""
        if self.big_ctas == 0:
            return self.grid, self.blocks_per_cta
        return self.big_ctas, self.tail_blocks

    def piece_starts(self) -> np.ndarray:
        """First global block of every piece, int64 [grid]."""
        big, tail = self.pieces()
        index = np.arange(self.grid, dtype=np.int64)
        return np.where(index < big, index * self.blocks_per_cta, big * self.blocks_per_cta + (index - big) * tail)


# Row-switch cost of the decode kernel in blocks streamed (measured on B200);
# the environment override is for tuning sweeps.
ROW_COST = float(os.environ.get("PKV_DECODE_ROW_COST", "3.0"))


def decode_tables(prefix: np.ndarray, grid: int, weights: np.ndarray | None = None,
                  row_cost: float = ROW_COST) -> tuple[np.ndarray, np.ndarray]:
    """Piece tables of a batch (host): pieces int32 [grid, 4], row_pieces int32 [B, 2].

    ``prefix`` int32 [B + 1] (prefix[0] == 0); see pkv_decode_tables.
    """
    prefix = np.ascontiguousarray(prefix, dtype=np.int32)
    batch = len(prefix) - 1
    pieces = np.empty((grid, 4), dtype=np.int32)
    row_pieces = np.empty((batch, 2), dtype=np.int32)
    if weights is not None:
        weights = np.ascontiguousarray(weights, dtype=np.float32)
        if weights.shape != (grid,):
            raise ValueError("weights must hold one value per piece")
    check(
        lib.pkv_decode_tables(
            prefix.ctypes.data,
            batch,
            grid,
            None if weights is None else weights.ctypes.data,
            row_cost,
            pieces.ctypes.data,
            row_pieces.ctypes.data,
        )
    )
    return pieces, row_pieces


def decode_plan(device: torch.device, batch: int, total_blocks: int) -> DecodePlan:
    grid = ctypes.c_int32()
    per_cta = ctypes.c_int32()
    big = ctypes.c_int32()
    tail = ctypes.c_int32()
    workspace = ctypes.c_int64()
    index = device.index if device.index is not None else torch.cuda.current_device()
    check(
        lib.pkv_decode_plan(
            index,
            batch,
            total_blocks,
            ctypes.byref(grid),
            ctypes.byref(per_cta),
            ctypes.byref(big),
            ctypes.byref(tail),
            ctypes.byref(workspace),
        )
    )
    return DecodePlan(grid.value, per_cta.value, workspace.value, big.value, tail.value)


def decode_slots(device: torch.device) -> int:
    """The largest grid ``decode_plan`` chooses on ``device`` (resident CTA slots)."""
    return decode_plan(device, 1, 1 << 24).grid


def decode_attention(
    pool: Tensor,
    layer: int,
    query: Tensor,
    lengths: Tensor,
    prefix: Tensor,
    flat: Tensor,
    total_blocks: int,
    plan: DecodePlan,
    out: Tensor,
    workspace: Tensor | None,
    error_flag: Tensor,
    pieces: Tensor | None = None,
    row_pieces: Tensor | None = None,
) -> Tensor:
    """Split-K block-table attention of FP16 query [B, 32, 64] into ``out``."""
    device = pool.device
    batch = query.shape[0]
    if query.ndim != 3 or query.shape[1:] != (_QUERY_HEADS, _HEAD_DIM) or query.dtype != torch.float16:
        raise ValueError("query must be FP16 [batch, 32, 64]")
    if query.stride()[1:] != (_HEAD_DIM, 1):
        query = query.contiguous()
    if out.shape != query.shape or out.dtype != torch.float16 or out.stride()[1:] != (_HEAD_DIM, 1):
        raise ValueError("out must be FP16 [batch, 32, 64] with contiguous rows")
    for name, tensor in (("query", query), ("out", out), ("lengths", lengths), ("prefix", prefix), ("flat", flat)):
        _require_cuda(name, tensor, device)
    check(
        lib.pkv_decode_attention(
            _ptr(pool),
            pool.shape[2],
            layer,
            _ptr(query),
            query.stride(0),
            _ptr(lengths),
            _ptr(prefix),
            _ptr(flat),
            _ptr(pieces),
            _ptr(row_pieces),
            batch,
            total_blocks,
            plan.grid,
            plan.blocks_per_cta,
            *plan.pieces(),
            _ptr(out),
            out.stride(0),
            _ptr(workspace),
            0 if workspace is None else workspace.numel() * workspace.element_size(),
            _ptr(error_flag),
            _stream(device),
        )
    )
    return out


def prefill_attention(
    pool: Tensor, layer: int, query: Tensor, blocks: Tensor, start: int, out: Tensor, error_flag: Tensor
) -> Tensor:
    """Causal attention of a prompt chunk's rotated FP16 query [T, 32, 64] into ``out``.

    Token t of the chunk sits at position ``start + t`` and attends to
    positions 0 .. start + t through ``blocks`` (int32, the request's physical
    block per 16 positions); the chunk's K/V must already be in the pool.
    """
    device = pool.device
    if query.ndim != 3 or query.shape[1:] != (_QUERY_HEADS, _HEAD_DIM) or query.dtype != torch.float16:
        raise ValueError("query must be FP16 [tokens, 32, 64]")
    if query.stride()[1:] != (_HEAD_DIM, 1):
        query = query.contiguous()
    if out.shape != query.shape or out.dtype != torch.float16 or out.stride()[1:] != (_HEAD_DIM, 1):
        raise ValueError("out must be FP16 [tokens, 32, 64] with contiguous rows")
    tokens = query.shape[0]
    if blocks.dtype != torch.int32 or blocks.ndim != 1 or blocks.numel() * 16 < start + tokens:
        raise ValueError("blocks must be int32 with one entry per 16 positions of the chunk's request")
    for name, tensor in (("query", query), ("out", out), ("blocks", blocks)):
        _require_cuda(name, tensor, device)
    check(
        lib.pkv_prefill_attention(
            _ptr(pool), pool.shape[2], layer, _ptr(query), query.stride(0), _ptr(blocks), start, tokens,
            _ptr(out), out.stride(0), _ptr(error_flag), _stream(device),
        )
    )
    return out


def decode_layer(
    pool: Tensor,
    layer: int,
    query: Tensor,
    key: Tensor,
    value: Tensor,
    rope_table: Tensor,
    lengths: Tensor,
    prefix: Tensor,
    flat: Tensor,
    total_blocks: int,
    plan: DecodePlan,
    out: Tensor,
    workspace: Tensor | None,
    error_flag: Tensor,
    pieces: Tensor | None = None,
    row_pieces: Tensor | None = None,
) -> Tensor:
    """Fused decode layer of a staged batch: RoPE(Q, K), new-token KV write, attention.

    query [B, 32, 64] unrotated, key/value [B, 4, 64] for the new tokens at
    positions lengths-1 (the staged view); writes attention to ``out``.
    """
    batch = query.shape[0]
    if query.shape[1:] != (_QUERY_HEADS, _HEAD_DIM) or query.stride()[1:] != (_HEAD_DIM, 1):
        raise ValueError("query must be FP16 [batch, 32, 64] with contiguous rows")
    if key.shape != (batch, _KV_HEADS, _HEAD_DIM) or value.shape != key.shape:
        raise ValueError("K and V must share FP16 [batch, 4, 64] on the pool device")
    if key.stride()[1:] != (_HEAD_DIM, 1) or value.stride() != key.stride():
        key, value = key.contiguous(), value.contiguous()
    for name, tensor in (("query", query), ("key", key), ("value", value)):
        if tensor.dtype != torch.float16:
            raise ValueError(f"{name} must be FP16")
    if out.shape != query.shape or out.dtype != torch.float16 or out.stride()[1:] != (_HEAD_DIM, 1):
        raise ValueError("out must be FP16 [batch, 32, 64] with contiguous rows")
    check(
        lib.pkv_decode_layer(
            _ptr(pool),
            pool.shape[2],
            layer,
            _ptr(query),
            query.stride(0),
            _ptr(key),
            _ptr(value),
            key.stride(0),
            _ptr(rope_table),
            _ptr(lengths),
            _ptr(prefix),
            _ptr(flat),
            _ptr(pieces),
            _ptr(row_pieces),
            batch,
            total_blocks,
            plan.grid,
            plan.blocks_per_cta,
            *plan.pieces(),
            _ptr(out),
            out.stride(0),
            _ptr(workspace),
            0 if workspace is None else workspace.numel() * workspace.element_size(),
            _ptr(error_flag),
            0,  # flags
            _stream(pool.device),
        )
    )
    return out


@dataclass(frozen=True, slots=True)
class SplitSums:
    """The output of a split-K linear layer before its splits are added:
    FP32 partial sums [splits, rows, n].  Consumers add the splits in order
    and round once to FP16, where the FP16 GEMM output would have been."""

    partials: Tensor

    @property
    def splits(self) -> int:
        return self.partials.shape[0]

    @property
    def shape(self) -> tuple[int, int]:
        return self.partials.shape[1], self.partials.shape[2]

    def to_half(self, out: Tensor | None = None) -> Tensor:
        """fp16(sum of the splits) as [rows, n] (``pkv_split_sum``)."""
        rows, n = self.shape
        if out is None:
            out = torch.empty((rows, n), dtype=torch.float16, device=self.partials.device)
        check(lib.pkv_split_sum(_ptr(self.partials), self.splits, rows, n, _ptr(out), out.stride(0),
                                _stream(self.partials.device)))
        return out


def add_rms_norm(hidden: Tensor, delta: Tensor | SplitSums | None, weight: Tensor, out: Tensor,
                 eps: float = 1e-5) -> Tensor:
    """``hidden += delta`` (FP16, in place, when given), then ``out = rms_norm(hidden) * weight``.

    hidden, delta, out FP16 [rows, dim] contiguous; weight FP16 [dim].  Same
    rounding points as dense.rms_norm after an FP16 residual add.  ``delta``
    may be a linear layer's ``SplitSums``: its splits are added and rounded
    to FP16 in the same kernel.
    """
    rows, dim = hidden.shape
    if isinstance(delta, SplitSums):
        if delta.shape != (rows, dim) or delta.partials.dtype != torch.float32:
            raise ValueError("delta must hold FP32 split sums [splits, rows, dim]")
        for name, tensor, shape in (("hidden", hidden, (rows, dim)), ("out", out, (rows, dim)),
                                    ("weight", weight, (dim,))):
            if tensor.shape != shape or tensor.dtype != torch.float16 or not tensor.is_contiguous():
                raise ValueError(f"{name} must be contiguous FP16 {list(shape)}")
            _require_cuda(name, tensor, hidden.device)
        check(lib.pkv_add_rms_norm_split(_ptr(hidden), _ptr(delta.partials), delta.splits, _ptr(weight), _ptr(out),
                                         rows, dim, eps, _stream(hidden.device)))
        return out
    for name, tensor, shape in (("hidden", hidden, (rows, dim)), ("out", out, (rows, dim)),
                                ("weight", weight, (dim,)), ("delta", delta, (rows, dim))):
        if tensor is None:
            continue
        if tensor.shape != shape or tensor.dtype != torch.float16 or not tensor.is_contiguous():
            raise ValueError(f"{name} must be contiguous FP16 {list(shape)}")
        _require_cuda(name, tensor, hidden.device)
    check(lib.pkv_add_rms_norm(_ptr(hidden), _ptr(delta), _ptr(weight), _ptr(out), rows, dim, eps,
                               _stream(hidden.device)))
    return out


def silu_mul(gate_up: Tensor | SplitSums, out: Tensor | None = None) -> Tensor:
    """``silu(gate) * up`` of FP16 gate_up [rows, 2 * inter] (gate first) into [rows, inter].

    ``gate_up`` may be the gate/up layer's ``SplitSums``, added in the same kernel.
    """
    if isinstance(gate_up, SplitSums):
        rows, width = gate_up.shape
        if out is None:
            out = torch.empty((rows, width // 2), dtype=torch.float16, device=gate_up.partials.device)
        check(lib.pkv_silu_mul_split(_ptr(gate_up.partials), gate_up.splits, _ptr(out), rows, width // 2,
                                     _stream(gate_up.partials.device)))
        return out
    rows, width = gate_up.shape
    if gate_up.dtype != torch.float16 or not gate_up.is_contiguous() or width % 2:
        raise ValueError("gate_up must be contiguous FP16 [rows, 2 * inter]")
    if out is None:
        out = torch.empty((rows, width // 2), dtype=torch.float16, device=gate_up.device)
    check(lib.pkv_silu_mul(_ptr(gate_up), _ptr(out), rows, width // 2, _stream(gate_up.device)))
    return out


# Rows up to which ``linear`` uses the matrix-vector kernel.  Measured on
# B200 against the library GEMM, weights read from DRAM: at one row it takes
# 4.6-9.2 us against 7.4-17.3 us on the decoder's Q/K/V, output and down
# projections, about the same on gate/up and the LM head; from two rows on it
# turns CUDA-core bound.
GEMV_MAX_ROWS = 1
# Rows up to which ``linear`` uses the tcgen05 split-K kernel.  The kernel
# takes up to 256 rows (its MMA N limit); measured on B200 over 22 layers of the
# decoder step's projections, norms and SwiGLU product replayed as one graph,
# it is ahead of the library GEMM at 8 rows (39.8 against 46.1 us per layer),
# even with it at 16-32 (40.4 against 39.5, 40.3 against 40.1) and behind from
# 64 rows (46 against 41 at 64, 69 against 47 at 256).
TC_MAX_ROWS = 32

_linear_errors: dict[int, Tensor] = {}


def linear_error_flag(device: torch.device) -> Tensor:
    """The device error flag of this device's ``pkv_linear`` launches (int32, zero when all is well)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    flag = _linear_errors.get(index)
    if flag is None:
        with torch.inference_mode(False):
            flag = _linear_errors[index] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
    return flag


def linear_splits(rows: int, n: int, k: int) -> int:
    """The K split ``pkv_linear`` uses for this shape on the current device."""
    splits = ctypes.c_int32()
    check(lib.pkv_linear_splits(rows, n, k, ctypes.byref(splits)))
    return splits.value


def _tc_shape_ok(x: Tensor, weight: Tensor) -> bool:
    rows, k = x.shape
    n = weight.shape[0]
    return (
        GEMV_MAX_ROWS < rows <= TC_MAX_ROWS
        and n % 128 == 0
        and k % 64 == 0
        and x.dtype == torch.float16
        and weight.dtype == torch.float16
        and weight.shape == (n, k)
        and weight.is_contiguous()
        and x.stride(1) == 1
        and x.stride(0) % 8 == 0
        and x.data_ptr() % 16 == 0
        and weight.data_ptr() % 16 == 0
    )


def linear(x: Tensor, weight: Tensor, out: Tensor | None = None, *, split_sums: bool = False) -> Tensor | SplitSums:
    """``F.linear(x, weight)`` for FP16 x [rows, k] and weight [n, k], no bias.

    One row runs this library's matrix-vector kernel (``pkv_gemv``, bound by
    reading the weight once); 2 to ``TC_MAX_ROWS`` rows its tcgen05 kernel
    (``pkv_linear``, split over K to cover the GPU); other shapes (more rows, k
    not a multiple of 64, n not of 128, unaligned or strided operands) the
    library GEMM.  All
    sum in FP32 and round once, in different orders.  With ``split_sums`` a
    split tcgen05 layer returns its ``SplitSums`` for a fused consumer
    (``add_rms_norm``, ``silu_mul``) instead of adding them here.
    """
    rows, k = x.shape
    n = weight.shape[0]
    if _tc_shape_ok(x, weight):
        splits = linear_splits(rows, n, k)
        flag = linear_error_flag(x.device)
        if splits > 1:
            partials = torch.empty((splits, rows, n), dtype=torch.float32, device=x.device)
            check(lib.pkv_linear(_ptr(x), x.stride(0), _ptr(weight), rows, n, k, splits, None, 0, _ptr(partials),
                                 _ptr(flag), _stream(x.device)))
            sums = SplitSums(partials)
            return sums if split_sums and out is None else sums.to_half(out)
        if out is None:
            out = torch.empty((rows, n), dtype=torch.float16, device=x.device)
        check(lib.pkv_linear(_ptr(x), x.stride(0), _ptr(weight), rows, n, k, 1, _ptr(out), out.stride(0), None,
                             _ptr(flag), _stream(x.device)))
        return out
    if (
        rows > GEMV_MAX_ROWS
        or k % 8
        or x.dtype != torch.float16
        or weight.dtype != torch.float16
        or weight.shape != (n, k)
        or not weight.is_contiguous()
        or x.stride(1) != 1
        or x.stride(0) % 8
        or x.data_ptr() % 16
        or weight.data_ptr() % 16
    ):
        result = torch.nn.functional.linear(x, weight)
        if out is None:
            return result
        out.copy_(result)
        return out
    if out is None:
        out = torch.empty((rows, n), dtype=torch.float16, device=x.device)
    check(lib.pkv_gemv(_ptr(x), x.stride(0), _ptr(weight), rows, n, k, _ptr(out), out.stride(0), _stream(x.device)))
    return out
