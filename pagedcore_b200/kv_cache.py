"""Drop-in KV pool and allocator for PagedCore's paged KV path on B200.

Same API, argument meaning and exception contract as
src/pagedcore/kv_cache.py: ``allocate_kv_pool`` (17-47) and ``KVAllocator``
(63-357).  The bookkeeping lives in the C++ ledger (``csrc/ledger.cpp``) and
every K/V write is the sm_100a scatter kernel (``csrc/append_kv.cu``); this
module only validates arguments in the reference's order, maps request ids to
ledger handles and passes device pointers across the C ABI.

Differences from the reference, by design:
- the pool must be CUDA storage (the reference also accepts CPU pools for its
  own allocator tests; the bookkeeping alone is :class:`BlockLedger`);
- ``validation="incremental"`` replaces the O(pool) re-validation on every
  call by a check of the touched requests (the default stays "full");
- batched entry points for the decode hot path: ``write_decode_batch``,
  ``append(..., rotate=True)`` with K-RoPE fused, and ``decode_batch`` which
  returns the device-side block tables of a batch.
"""

from __future__ import annotations

from collections.abc import Iterator, Sequence
from contextlib import contextmanager
from dataclasses import dataclass
from threading import current_thread

import numpy as np
import torch
from torch import Tensor

from pagedcore_b200 import kernels
from pagedcore_b200._lib import VIEW_STAGED as _VIEW_STAGED
from pagedcore_b200._lib import check, device_error_message, lib
from pagedcore_b200.config import PagedCoreConfig
from pagedcore_b200.engine_types import BlockId, BlockTable, CapacityCounts, KVReservation, RequestId
from pagedcore_b200.ledger import BlockLedger
from pagedcore_b200.rope import device_table

_LAYERS = 22
_BLOCK_TOKENS = 16
_UNKNOWN_BASE = -(1 << 62)


def allocate_kv_pool(config: PagedCoreConfig, *, device: str | torch.device = "cuda:0") -> Tensor:
    """Allocate the FP16 [22, 2, blocks, 16, 4, 64] pool once (kv_cache.py:17-47).

    Storage is uninitialised: only written, valid slots may be read.
    """
    target = torch.device(device)
    if target.type != "cuda":
        raise ValueError("KV pool requires a CUDA device")
    if not torch.cuda.is_available():
        raise RuntimeError("KV pool requires an available CUDA runtime")
    pool_bytes = config.kv_pool_mib * 2**20
    margin_bytes = config.workspace_margin_mib * 2**20
    block_bytes = _LAYERS * 2 * config.block_tokens * 4 * 64 * 2
    num_blocks = pool_bytes // block_bytes
    free_bytes, _ = torch.cuda.mem_get_info(target)
    if free_bytes < pool_bytes + margin_bytes:
        raise RuntimeError("configured KV pool and workspace margin do not fit in GPU memory")
    pool = torch.empty(
        (_LAYERS, 2, num_blocks, config.block_tokens, 4, 64), dtype=torch.float16, device=target
    )
    if torch.cuda.mem_get_info(target)[0] < margin_bytes:
        del pool
        raise RuntimeError("KV pool allocation leaves less than the configured workspace margin")
    return pool


@dataclass(slots=True)
class DecodeBatch:
    """Device-resident block tables of a batch: what the attention kernels read.

    Views of one int32 device buffer, in this order: ``pieces`` [grid][4]
    (begin, end, first row and its first block of each CTA's piece),
    ``row_pieces`` [B][2] (first and last piece of each row), ``lengths``
    [B], ``prefix`` [B+1] (cumulative block counts) and ``flat`` (the
    concatenated block tables).
    """

    requests: tuple[RequestId, ...]
    lengths: Tensor
    prefix: Tensor
    flat: Tensor
    pieces: Tensor
    row_pieces: Tensor
    total_blocks: int
    plan: kernels.DecodePlan
    host_lengths: np.ndarray


@dataclass(slots=True)
class _Staged:
    requests: tuple[RequestId, ...]
    handles: np.ndarray
    rows: dict[RequestId, int]
    slots: Tensor  # int32 device [B]
    positions: Tensor  # int32 device [B]
    host_positions: np.ndarray
    written: int = 0  # layers written for every row by write_decode_batch / decode_layer
    batch: DecodeBatch | None = None
    staged_batch: DecodeBatch | None = None  # staged view of every row, for decode_layer
    launch_args: tuple | None = None  # fixed pkv_decode_layer arguments of this step
    flat_capacity: int = 0  # room of the flat block list in the step's upload buffer (a bound on total)


@dataclass(slots=True)
class _UploadSlot:
    host: Tensor  # pinned int32
    device: Tensor  # int32 on the pool device
    copied: torch.cuda.Event  # the host -> device copy into ``device`` has finished
    released: torch.cuda.Event  # the last kernel reading ``device`` has finished
    used: bool = False


class _StepUploads:
    """Per-step int32 tables, copied to the device on a side stream.

    Two slots alternate: the tables of step i+1 are written and copied while
    step i's kernels still read the other slot, so the copy is done when the
    compute stream reaches step i+1 and its wait costs nothing.  A slot is
    reused only after the compute stream has passed the step that read it.
    """

    def __init__(self, device: torch.device, compute: torch.cuda.Stream) -> None:
        self._device = device
        self._compute = compute
        self._copy = torch.cuda.Stream(device)
        self._slots: list[_UploadSlot] = []
        self._next = 0

    def _ensure(self, count: int) -> None:
        if self._slots and self._slots[0].host.numel() >= count:
            return
        # Growing: no copy or kernel may still use the old buffers.
        torch.cuda.synchronize(self._device)
        size = max(count, 2 * self._slots[0].host.numel() if self._slots else 8192)
        with torch.inference_mode(False):  # persistent buffers, updated in place in any mode
            self._slots = [
                _UploadSlot(
                    torch.empty(size, dtype=torch.int32, pin_memory=True),
                    torch.empty(size, dtype=torch.int32, device=self._device),
                    torch.cuda.Event(),
                    torch.cuda.Event(),
                )
                for _ in range(2)
            ]
        self._next = 0

    def upload(self, arrays: Sequence[np.ndarray]) -> tuple[Tensor, _UploadSlot]:
        count = sum(len(a) for a in arrays)
        self._ensure(count)
        slot = self._slots[self._next]
        self._next ^= 1
        if slot.used:
            slot.copied.synchronize()  # its pinned buffer is no longer being read
            self._copy.wait_event(slot.released)  # nor its device buffer
        view = slot.host.numpy()
        offset = 0
        for array in arrays:
            view[offset : offset + len(array)] = array
            offset += len(array)
        with torch.cuda.stream(self._copy):
            slot.device[:count].copy_(slot.host[:count], non_blocking=True)
        slot.copied.record(self._copy)
        self._compute.wait_event(slot.copied)
        slot.used = True
        return slot.device[:count], slot

    def release(self, slot: _UploadSlot) -> None:
        """Every kernel reading the slot has been enqueued on the compute stream."""
        slot.released.record(self._compute)


class PrefillAppend:
    """One planned prompt chunk of ``KVAllocator.prefill_append``."""

    def __init__(self, allocator: KVAllocator, blocks: np.ndarray, device_blocks: Tensor, slots: Tensor,
                 positions: Tensor, start: int, tokens: int) -> None:
        self._allocator = allocator
        self._host_blocks = blocks
        self.blocks = device_blocks
        self.slots = slots
        self.positions = positions
        self.start = start
        self.tokens = tokens
        self._split_batch: DecodeBatch | None = None

    @torch.inference_mode()
    def write_layer(self, layer: int, key: Tensor, value: Tensor, query: Tensor, *, in_place: bool = False) -> Tensor:
        """Rotate K and write K/V [T, 4, 64] at `layer`; return Q [T, 32, 64] rotated.

        ``in_place=True`` rotates ``query`` itself (its [32, 64] rows must be
        contiguous; the token stride may be anything, e.g. a view of a fused
        Q/K/V projection) and returns it.
        """
        allocator = self._allocator
        allocator._check_worker()
        if type(layer) is not int or not 0 <= layer < _LAYERS:
            raise ValueError("layer_index must identify one of the 22 decoder layers")
        query_in = query.reshape(1, self.tokens, 32, 64)
        if in_place:
            if query.stride()[-2:] != (64, 1) or query_in.data_ptr() != query.data_ptr():
                raise ValueError("in-place rotation needs query rows of contiguous [32, 64] heads")
            rotated = query_in
        else:
            rotated = torch.empty((1, self.tokens, 32, 64), dtype=torch.float16, device=allocator._pool.device)
        kernels.append_kv(
            allocator._pool, key.reshape(1, self.tokens, 4, 64), value.reshape(1, self.tokens, 4, 64), self.slots,
            layer_begin=layer, error_flag=allocator._error, positions=self.positions, rope_table=allocator._rope,
            query_in=query_in, query_out=rotated,
        )
        return rotated[0]

    @torch.inference_mode()
    def attend(self, layer: int, query: Tensor, out: Tensor | None = None) -> Tensor:
        """Causal attention [T, 32, 64] of the rotated chunk queries at `layer` over the pool.

        One launch of the prefill kernel (``pkv_prefill_attention``): every
        16-token query tile streams the request's blocks once.
        """
        allocator = self._allocator
        allocator._check_worker()
        if type(layer) is not int or not 0 <= layer < _LAYERS:
            raise ValueError("layer_index must identify one of the 22 decoder layers")
        if out is None:
            out = torch.empty(query.shape, dtype=torch.float16, device=allocator._pool.device)
        return kernels.prefill_attention(allocator._pool, layer, query, self.blocks, self.start, out, allocator._error)

    @torch.inference_mode()
    def attend_split(self, layer: int, query: Tensor, out: Tensor | None = None) -> Tensor:
        """The same attention through the split-K decode kernel, token t as a row of length start + t + 1."""
        if self._split_batch is None:
            self._split_batch = self._allocator._prefill_batch(self._host_blocks, self.start, self.tokens)
        return self._allocator.attend(self._split_batch, query, layer_index=layer, out=out)


def padded_tables(
    pieces: np.ndarray, row_pieces: np.ndarray, host: np.ndarray, count: int, total: int, rows: int, grid: int
) -> np.ndarray:
    """A batch's step tables in the padded layout of ``rows`` rows and ``grid`` pieces.

    pieces [p][4] and row_pieces [count][2] from ``kernels.decode_tables``;
    host = lengths [count] | prefix [count + 1] | flat [total].  Layout:
    pieces [grid][4] | row_pieces [rows][2] | lengths [rows] | prefix [rows + 1]
    | flat [total], padded with empty pieces (0, 0, 0, 0), rows without pieces
    (0, 0), length 0 and prefix ``total``, which every kernel skips.
    """
    if count > rows or len(pieces) > grid:
        raise ValueError(f"the batch needs {count} rows and {len(pieces)} pieces; the layout has {rows} and {grid}")
    tables = np.zeros(4 * grid + 4 * rows + 1 + total, dtype=np.int32)
    tables[: 4 * len(pieces)] = pieces.reshape(-1)
    at = 4 * grid
    tables[at : at + 2 * count] = row_pieces.reshape(-1)
    at += 2 * rows
    tables[at : at + count] = host[:count]  # lengths
    at += rows
    tables[at : at + count + 1] = host[count : 2 * count + 1]  # prefix
    tables[at + count + 1 : at + rows + 1] = total
    tables[at + rows + 1 :] = host[2 * count + 1 : 2 * count + 1 + total]  # flat
    return tables


@dataclass(slots=True)
class _SlotSpeeds:
    """Per-CTA-slot weights of the decode pieces, from measured wall times."""

    weights: np.ndarray  # float32 [grid], mean 1
    updates: int = 0
    pending: tuple | None = None  # (pinned counters [grid * 4], event) of a finished step


_SPEED_UPDATES = 6  # weight updates before the weights freeze
_PIECES_PER_ROW_MAX = 8  # steps with more pieces per row than this are not measured


class KVAllocator:
    """Assign blocks within an existing CUDA pool (kv_cache.py:63-90).

    Construct and use on the model worker thread; CUDA work stays on the
    stream current at construction.  Block reads borrow pool storage.
    """

    def __init__(self, pool: Tensor, *, validation: str = "full", balance: str = "rows") -> None:
        if (
            pool.ndim != 6
            or pool.shape[:2] != (22, 2)
            or pool.shape[2] < 1
            or pool.shape[3:] != (16, 4, 64)
            or pool.dtype != torch.float16
            or pool.device.type not in ("cpu", "cuda")
            or not pool.is_contiguous()
            or pool.requires_grad
        ):
            raise ValueError("KV pool must be contiguous FP16 [22, 2, blocks, 16, 4, 64] storage")
        if pool.device.type != "cuda":
            raise ValueError("KV pool must be CUDA storage: the B200 KV path has no CPU implementation")
        self._pool = pool
        self._worker = current_thread()
        self._stream = torch.cuda.current_stream(pool.device)
        self._ledger = BlockLedger(pool.shape[2], validation)
        self._handles: dict[RequestId, int] = {}
        self._next_handle = 1
        self._staged: _Staged | None = None
        with torch.inference_mode(False):  # zeroed in place after a device error, in any mode
            self._error = torch.zeros(1, dtype=torch.int32, device=pool.device)
        self._rope = device_table(pool.device)
        self._workspace: Tensor | None = None
        self._uploads = _StepUploads(pool.device, self._stream)
        # How the decode pieces are cut: "rows" balances blocks plus row
        # switches (a function of the batch only); "measured" also weights each
        # CTA slot by its measured speed (slots on some SMs stream slower), the
        # weights learnt over the first staged steps and then frozen.
        if balance not in ("rows", "measured"):
            raise ValueError("balance must be 'rows' or 'measured'")
        self._balance = balance
        self._speeds: dict[int, _SlotSpeeds] = {}
        # Grid of every decode launch since the slot counters were last zeroed
        # (None: launches outside a measured step, or of mixed grids).
        self._window_grid: int | None = None

    # -- plumbing -------------------------------------------------------------
    @property
    def pool(self) -> Tensor:
        return self._pool

    @property
    def ledger(self) -> BlockLedger:
        return self._ledger

    def _check_worker(self) -> None:
        if current_thread() is not self._worker:
            raise RuntimeError("KV allocator must be used by its owning model worker")
        if torch.cuda.current_stream(self._pool.device) != self._stream:
            raise RuntimeError("KV allocator must use its owning CUDA stream")

    def _handle(self, request_id: RequestId, unknown_index: int = 0) -> int:
        handle = self._handles.get(request_id)
        return handle if handle is not None else _UNKNOWN_BASE - unknown_index

    def _call(self, function, request_id: RequestId | None, *args):
        try:
            return function(*args)
        except KeyError:
            raise KeyError(request_id) from None

    def _upload_i32(self, *arrays: np.ndarray) -> Tensor:
        """One pinned host->device copy of several int32 arrays, concatenated."""
        host = torch.empty(sum(len(a) for a in arrays), dtype=torch.int32, pin_memory=True)
        view = host.numpy()
        offset = 0
        for array in arrays:
            view[offset : offset + len(array)] = array
            offset += len(array)
        return host.to(self._pool.device, non_blocking=True)

    def _workspace_for(self, nbytes: int) -> Tensor | None:
        if nbytes <= 0:
            return None
        if self._workspace is None or self._workspace.numel() * 4 < nbytes:
            with torch.inference_mode(False):  # persistent, updated in place in any mode
                self._workspace = torch.zeros((nbytes + 3) // 4, dtype=torch.float32, device=self._pool.device)
        return self._workspace

    # -- per-slot speed weights (balance="measured") ------------------------------
    def _slot_counters(self, plan: kernels.DecodePlan) -> Tensor | None:
        """The plan's [grid * 4] uint32 wall-time counters (after the claim counters), as int32."""
        workspace = self._workspace_for(plan.workspace_bytes)
        if workspace is None:
            return None
        start = kernels.CLAIM_BYTES // 4
        return workspace[start : start + 4 * plan.grid].view(torch.int32)

    def _slot_weights(self, plan: kernels.DecodePlan) -> np.ndarray | None:
        if self._balance != "measured" or plan.grid < 2:
            return None
        state = self._speeds.get(plan.grid)
        if state is None:
            state = self._speeds[plan.grid] = _SlotSpeeds(np.ones(plan.grid, dtype=np.float32))
            self._reset_slot_counters(plan.grid)  # the first measured step starts from zero
        if state.pending is not None and state.pending[1].query():
            counters = state.pending[0].numpy().astype(np.uint32).reshape(plan.grid, 4)
            seconds = counters.max(axis=1).astype(np.float64)
            state.pending = None
            if seconds.min() > 0:
                # Give a slot more work the sooner it finished (damped), mean 1.
                step = (seconds.mean() / seconds) ** 0.7
                weights = np.clip(state.weights * step, 0.5, 2.0)
                state.weights = (weights / weights.mean()).astype(np.float32)
                state.updates += 1
        return state.weights

    def _reset_slot_counters(self, grid: int) -> None:
        """Zero every slot's counters: the next window holds launches of ``grid`` only."""
        if self._workspace is not None:
            start = kernels.CLAIM_BYTES // 4
            self._workspace[start : start + 4 * kernels.decode_slots(self._pool.device)].zero_()
        self._window_grid = grid

    def _measure_slots(self, plan: kernels.DecodePlan, rows: int) -> None:
        """After a staged step of ``rows`` rows: copy out and clear its slot counters while calibrating.

        A measurement covers only steps of the plan's grid: launches of another
        grid add to the same counters (a smaller grid's partials may even
        overwrite them), so a step of another grid, or attention launched
        outside a staged step, starts the window over.  Steps with fewer than
        one row per _PIECES_PER_ROW_MAX pieces are not measured: there each
        row spans many pieces and a slot's time reflects where the row
        boundaries fall in this batch more than its SM's speed.
        """
        if self._balance != "measured":
            return
        if rows * _PIECES_PER_ROW_MAX < plan.grid:
            self._window_grid = None
            return
        if self._window_grid != plan.grid:
            self._reset_slot_counters(plan.grid)
            return
        if plan.grid < 2:
            return
        state = self._speeds.get(plan.grid)
        counters = self._slot_counters(plan)
        if state is None or counters is None or state.updates >= _SPEED_UPDATES or state.pending is not None:
            return
        host = torch.empty(counters.shape, dtype=torch.int32, pin_memory=True)
        host.copy_(counters, non_blocking=True)
        done = torch.cuda.Event()
        done.record(self._stream)
        counters.zero_()
        state.pending = (host, done)

    def slot_weights(self) -> dict[int, np.ndarray]:
        """The measured per-slot weights by grid size (balance="measured")."""
        return {grid: state.weights.copy() for grid, state in self._speeds.items()}

    def check_device_errors(self) -> None:
        """Synchronise and raise if a kernel flagged an out-of-range block or position."""
        flag = int(self._error.item())
        if flag:
            self._error.zero_()
            raise RuntimeError(device_error_message(flag))

    # -- reference API ----------------------------------------------------------
    def create(self, reservation: KVReservation) -> None:
        """Grant credits at admission without assigning blocks (kv_cache.py:92-110)."""
        self._check_worker()
        request_id = reservation.request_id
        handle = self._handles.get(request_id)
        if handle is None:
            handle = self._next_handle
        self._ledger.reserve(handle, reservation.maximum_block_credits)
        if request_id not in self._handles:
            self._handles[request_id] = handle
            self._next_handle += 1

    def capacity(self) -> CapacityCounts:
        self._check_worker()
        return CapacityCounts(*self._ledger.capacity())

    def block_table(self, request_id: RequestId) -> BlockTable:
        self._check_worker()
        table = self._call(self._ledger.table, request_id, self._handle(request_id))
        return tuple(BlockId(block) for block in table)

    def cached_length(self, request_id: RequestId) -> int:
        self._check_worker()
        return self._call(self._ledger.length, request_id, self._handle(request_id))

    @torch.inference_mode()
    def append(self, request_id: RequestId, key: Tensor, value: Tensor, *, rotate: bool = False) -> None:
        """Append rotated K and unrotated V, each FP16 [22, tokens, 4, 64] (kv_cache.py:127-179).

        With ``rotate=True`` K is given unrotated and the kernel applies RoPE at
        the absolute positions it is written to.  A failed launch leaves
        ownership and valid positions unchanged.
        """
        self._check_worker()
        if self._ledger.staging:
            raise RuntimeError("KV mutation is not allowed during a staged decode append")
        handle = self._handle(request_id)
        self._call(self._ledger.length, request_id, handle)
        if (
            key.ndim != 4
            or key.shape[0] != 22
            or key.shape[1] < 1
            or key.shape[2:] != (4, 64)
            or value.shape != key.shape
            or key.dtype != torch.float16
            or value.dtype != torch.float16
            or key.device != self._pool.device
            or value.device != self._pool.device
        ):
            raise ValueError("K and V must share FP16 [22, tokens, 4, 64] on the pool device")
        tokens = key.shape[1]
        slots, start = self._call(self._ledger.append_plan, request_id, handle, tokens)
        if rotate:
            positions = np.arange(start, start + tokens, dtype=np.int32)
            meta = self._upload_i32(slots, positions)
            kernels.append_kv(
                self._pool, key, value, meta[:tokens], layer_begin=0, error_flag=self._error,
                positions=meta[tokens:], rope_table=self._rope,
            )
        else:
            meta = self._upload_i32(slots)
            kernels.append_kv(self._pool, key, value, meta, layer_begin=0, error_flag=self._error)
        # Publish valid positions only after both K and V writes were issued.
        self._ledger.append_commit(handle, tokens)

    @torch.inference_mode()
    def append_many(
        self,
        request_ids: Sequence[RequestId],
        key: Tensor,
        value: Tensor,
        tokens: Sequence[int],
        *,
        rotate: bool = False,
    ) -> None:
        """``append`` for several requests in one kernel launch.

        key/value FP16 [22, sum(tokens), 4, 64] hold the requests' tokens
        concatenated in request order (``tokens[i]`` positions for request i).
        Same slots and pool bytes as calling ``append`` for each request in
        order, and all or nothing: if any request's append would fail, no
        request changes.  Requests must be distinct.
        """
        self._check_worker()
        if self._ledger.staging:
            raise RuntimeError("KV mutation is not allowed during a staged decode append")
        request_ids = tuple(request_ids)
        counts = [int(t) for t in tokens]
        if not request_ids or len(counts) != len(request_ids):
            raise ValueError("append_many takes one token count per request")
        missing = next((request_id for request_id in request_ids if request_id not in self._handles), None)
        if missing is not None:
            raise KeyError(missing)
        handles = np.array([self._handles[request_id] for request_id in request_ids], dtype=np.int64)
        total = sum(counts)
        if (
            key.ndim != 4
            or key.shape[0] != 22
            or key.shape[1] != total
            or key.shape[2:] != (4, 64)
            or value.shape != key.shape
            or key.dtype != torch.float16
            or value.dtype != torch.float16
            or key.device != self._pool.device
            or value.device != self._pool.device
        ):
            raise ValueError("K and V must share FP16 [22, sum(tokens), 4, 64] on the pool device")
        slots, starts = self._ledger.append_plan_many(handles, counts)
        if rotate:
            positions = np.concatenate(
                [np.arange(start, start + count, dtype=np.int32) for start, count in zip(starts, counts, strict=True)]
            )
            meta = self._upload_i32(slots, positions)
            kernels.append_kv(
                self._pool, key, value, meta[:total], layer_begin=0, error_flag=self._error,
                positions=meta[total:], rope_table=self._rope,
            )
        else:
            meta = self._upload_i32(slots)
            kernels.append_kv(self._pool, key, value, meta, layer_begin=0, error_flag=self._error)
        # Publish every request only after the one launch was issued.
        self._ledger.append_commit_many(handles, counts)

    @contextmanager
    def prefill_append(self, request_id: RequestId, tokens: int) -> Iterator[PrefillAppend]:
        """Append a prompt chunk layer by layer, attending to it through the pool.

        Plans ``tokens`` new positions of ``request_id`` (blocks from the free
        list as ``append`` would take them) and yields a :class:`PrefillAppend`
        that writes one layer's K/V into those slots and computes that layer's
        causal attention from the pool pages.  The positions are published when
        the block exits without an error; otherwise nothing is published (the
        written slots stay unowned).
        """
        self._check_worker()
        if self._ledger.staging:
            raise RuntimeError("KV mutation is not allowed during a staged decode append")
        handle = self._handle(request_id)
        self._call(self._ledger.length, request_id, handle)
        if type(tokens) is not int or tokens < 1:
            raise ValueError("a prompt chunk needs at least one token")
        slots, start = self._call(self._ledger.append_plan, request_id, handle, tokens)
        existing = self._ledger.table(handle)
        # Physical block of every 16-token block of the extended context.
        blocks = np.asarray(
            [existing[j] if j < len(existing) else slots[16 * j - start] // 16
             for j in range(-(-(start + tokens) // 16))],
            dtype=np.int32,
        )
        positions = np.arange(start, start + tokens, dtype=np.int32)
        device = self._upload_i32(blocks, slots, positions)
        count = len(blocks)
        chunk = PrefillAppend(self, blocks, device[:count], device[count : count + tokens],
                              device[count + tokens :], start, tokens)
        yield chunk
        self._ledger.append_commit(handle, tokens)

    @contextmanager
    def append_decode(
        self, request_ids: tuple[RequestId, ...], *, layout: tuple[int, int] | None = None
    ) -> Iterator[None]:
        """Stage one token per request; commit all 22 layers together (kv_cache.py:181-219).

        ``layout=(rows, pieces)`` pads the staged step's device tables to
        ``rows`` rows and ``pieces`` pieces, so their addresses and a launch
        over them do not depend on the batch (``DecodeStepGraph``).
        """
        self._check_worker()
        if self._ledger.staging:
            raise RuntimeError("KV mutation is not allowed during a staged decode append")
        request_ids = tuple(request_ids)
        unknown = 0
        handles = np.empty(len(request_ids), dtype=np.int64)
        for row, request_id in enumerate(request_ids):
            handle = self._handles.get(request_id)
            if handle is None:
                unknown += 1
                handle = _UNKNOWN_BASE - unknown
            handles[row] = handle
        try:
            slots, positions = self._ledger.decode_begin(handles)
        except KeyError as error:
            missing = next((r for r in request_ids if r not in self._handles), None)
            raise KeyError(missing) from error
        count = len(request_ids)
        try:
            # The staged view (every row with its new token) is what the fused
            # decode layer reads; its tables travel with the slots in one copy.
            tables, total, plan = self._batch_tables(request_ids, handles, _VIEW_STAGED, layout)
            device, upload = self._uploads.upload((tables, slots, positions))
        except BaseException:
            self._ledger.decode_abort()
            raise
        rows, grid = (count, plan.grid) if layout is None else layout
        self._staged = _Staged(
            requests=request_ids,
            handles=handles,
            rows={request_id: row for row, request_id in enumerate(request_ids)},
            slots=device[len(tables) : len(tables) + count],
            positions=device[len(tables) + count :],
            host_positions=positions,
            staged_batch=self._device_batch(request_ids, tables, total, plan, device[: len(tables)], rows, grid),
            flat_capacity=upload.device.numel() - (4 * grid + 4 * rows + 1),
        )
        try:
            yield
        except BaseException:
            self._ledger.decode_abort()
            raise
        else:
            self._ledger.decode_commit()
            self._measure_slots(plan, count)
        finally:
            self._staged = None
            self._uploads.release(upload)

    @torch.inference_mode()
    def write_decode_layer(self, request_id: RequestId, layer_index: int, key: Tensor, value: Tensor) -> None:
        """Write one token's rotated K / unrotated V [4, 64], in layer order (kv_cache.py:221-246)."""
        self._check_worker()
        staged = self._staged
        layer = layer_index if type(layer_index) is int else -1
        handle = self._handle(request_id)
        self._call(self._ledger.decode_check, request_id, handle, layer)
        if any(
            tensor.shape != (4, 64) or tensor.dtype != torch.float16 or tensor.device != self._pool.device
            for tensor in (key, value)
        ):
            raise ValueError("K and V must share FP16 [4, 64] on the pool device")
        row = staged.rows[request_id]
        kernels.append_kv(
            self._pool, key[None, None], value[None, None], staged.slots[row : row + 1],
            layer_begin=layer, error_flag=self._error,
        )
        self._ledger.decode_mark(handle, layer)

    @torch.inference_mode()
    def write_decode_batch(
        self,
        layer_index: int,
        key: Tensor,
        value: Tensor,
        *,
        query: Tensor | None = None,
        rotate: bool = False,
    ) -> Tensor | None:
        """Batched ``write_decode_layer`` for every staged request, in staging order.

        key/value: FP16 [B, 4, 64] (unrotated K when ``rotate``).  With
        ``query`` [B, 32, 64] and ``rotate=True`` the rotated query is returned
        (RoPE of Q and K fused into the append kernel).
        """
        self._check_worker()
        staged = self._staged
        if staged is None:
            raise RuntimeError("decode writes require a staged append")
        layer = layer_index if type(layer_index) is int else -1
        self._ledger.decode_check(-1, layer)
        count = len(staged.requests)
        if key.shape != (count, 4, 64) or value.shape != key.shape:
            raise ValueError("K and V must share FP16 [batch, 4, 64] on the pool device")
        query_out = None
        if query is not None:
            if not rotate:
                raise ValueError("query is only accepted together with rotate=True")
            if query.shape != (count, 32, 64) or query.dtype != torch.float16:
                raise ValueError("query must be FP16 [batch, 32, 64]")
            query_out = torch.empty((1, count, 32, 64), dtype=torch.float16, device=self._pool.device)
        kernels.append_kv(
            self._pool,
            key[None],
            value[None],
            staged.slots,
            layer_begin=layer,
            error_flag=self._error,
            positions=staged.positions if rotate else None,
            rope_table=self._rope if rotate else None,
            query_in=None if query is None else query[None],
            query_out=query_out,
        )
        self._ledger.decode_mark(-1, layer)
        staged.written = layer + 1
        return None if query_out is None else query_out[0]

    @torch.inference_mode()
    def decode_layer(
        self, layer_index: int, query: Tensor, key: Tensor, value: Tensor, *, out: Tensor | None = None
    ) -> Tensor:
        """One decode layer of the staged batch in one launch.

        Fuses, for every staged row in staging order, ``write_decode_layer``
        of the new token (K given unrotated, rotated at the row's position),
        the RoPE of ``query`` and block-table attention over the row's
        context including the new token.  query FP16 [B, 32, 64] (unrotated),
        key/value FP16 [B, 4, 64]; returns the FP16 [B, 32, 64] attention.
        """
        self._check_worker()
        staged = self._staged
        if staged is None:
            raise RuntimeError("decode writes require a staged append")
        layer = layer_index if type(layer_index) is int else -1
        self._ledger.decode_check(-1, layer)
        count = len(staged.requests)
        if query.shape != (count, 32, 64) or query.dtype != torch.float16 or query.device != self._pool.device:
            raise ValueError("query must be FP16 [batch, 32, 64] on the pool device")
        if (
            key.shape != (count, 4, 64)
            or value.shape != key.shape
            or key.dtype != torch.float16
            or value.dtype != torch.float16
            or key.device != self._pool.device
            or value.device != self._pool.device
        ):
            raise ValueError("K and V must share FP16 [batch, 4, 64] on the pool device")
        if query.stride()[1:] != (64, 1):
            query = query.contiguous()
        if key.stride()[1:] != (64, 1) or value.stride() != key.stride():
            key, value = key.contiguous(), value.contiguous()
        if out is None:
            out = torch.empty((count, 32, 64), dtype=torch.float16, device=self._pool.device)
        elif out.shape != (count, 32, 64) or out.dtype != torch.float16 or out.stride()[1:] != (64, 1):
            raise ValueError("out must be FP16 [batch, 32, 64] with contiguous rows")
        fixed = staged.launch_args
        if fixed is None:
            batch = self.staged_decode_batch()
            fixed = staged.launch_args = self._decode_layer_args(batch, count, batch.plan.grid)
        pool_ptr, num_blocks, rope, lengths, prefix, flat, pieces, row_pieces, total, grid, per_cta, big, tail, ws, ws_bytes, \
            err, stream = fixed
        check(
            lib.pkv_decode_layer(
                pool_ptr, num_blocks, layer, query.data_ptr(), query.stride(0), key.data_ptr(), value.data_ptr(),
                key.stride(0), rope, lengths, prefix, flat, pieces, row_pieces, count, total, grid, per_cta, big, tail,
                out.data_ptr(), out.stride(0), ws, ws_bytes, err, 0, stream,
            )
        )
        self._ledger.decode_mark(-1, layer)
        staged.written = layer + 1
        return out

    def _decode_layer_args(self, batch: DecodeBatch, rows: int, grid: int) -> tuple:
        """Launch arguments of pkv_decode_layer that stay fixed for a staged step launched over
        ``rows`` rows and ``grid`` pieces (the batch's own, or its padded layout's)."""
        workspace = self._workspace_for(kernels.workspace_bytes(rows, grid))
        return (
            self._pool.data_ptr(), self._pool.shape[2], self._rope.data_ptr(), batch.lengths.data_ptr(),
            batch.prefix.data_ptr(), batch.flat.data_ptr(), batch.pieces.data_ptr(), batch.row_pieces.data_ptr(),
            batch.total_blocks,
            grid, batch.plan.blocks_per_cta, *batch.plan.pieces(),
            0 if workspace is None else workspace.data_ptr(),
            0 if workspace is None else workspace.numel() * 4, self._error.data_ptr(), self._stream.cuda_stream,
        )

    def staged_decode_batch(self) -> DecodeBatch:
        """Device tables of the staged batch with every row's new token included.

        Valid until the staged step ends (its buffer is reused two steps later).
        """
        staged = self._staged
        if staged is None:
            raise RuntimeError("decode writes require a staged append")
        if staged.staged_batch is None:
            staged.staged_batch = self._upload_batch(staged.requests, staged.handles, _VIEW_STAGED)
        return staged.staged_batch

    def decode_positions(self) -> np.ndarray:
        """RoPE positions (cached lengths before the append) of the staged rows."""
        if self._staged is None:
            raise RuntimeError("decode writes require a staged append")
        return self._staged.host_positions.copy()

    def iter_layer_blocks(self, request_id: RequestId, *, layer_index: int) -> Iterator[tuple[Tensor, Tensor]]:
        """Borrow valid [slots, 4, 64] pages, including a completed staged layer (kv_cache.py:248-270)."""
        self._check_worker()
        if type(layer_index) is not int or not 0 <= layer_index < _LAYERS:
            raise ValueError("layer_index must identify one of the 22 decoder layers")
        blocks, length = self._call(self._ledger.view, request_id, self._handle(request_id), layer_index)
        if length == 0:
            raise ValueError("attention requires a nonempty cache")
        for logical, physical in enumerate(blocks):
            self._check_worker()
            valid = min(_BLOCK_TOKENS, length - logical * _BLOCK_TOKENS)
            yield (
                self._pool[layer_index, 0, physical, :valid],
                self._pool[layer_index, 1, physical, :valid],
            )

    def read_block(self, request_id: RequestId, logical_block: int) -> tuple[Tensor, Tensor]:
        """Borrow K/V views [22, valid slots, 4, 64] of one logical block (kv_cache.py:272-284)."""
        self._check_worker()
        handle = self._handle(request_id)
        blocks = self._call(self._ledger.table, request_id, handle)
        length = self._ledger.length(handle)
        if type(logical_block) is not int or not 0 <= logical_block < len(blocks):
            raise ValueError("logical block must identify a cached block")
        physical = blocks[logical_block]
        valid = min(_BLOCK_TOKENS, length - logical_block * _BLOCK_TOKENS)
        return self._pool[:, 0, physical, :valid], self._pool[:, 1, physical, :valid]

    def release_all(self, request_id: RequestId) -> None:
        """Release once on the worker stream (kv_cache.py:286-298)."""
        self._check_worker()
        self._call(self._ledger.release, request_id, self._handle(request_id))
        del self._handles[request_id]

    # -- batched attention metadata ---------------------------------------------
    def decode_batch(self, request_ids: Sequence[RequestId], *, layer_index: int) -> DecodeBatch:
        """Device block tables, lengths and launch plan for a batch at ``layer_index``.

        During a staged decode the staged rows expose their new token once the
        layer was written.  The result is reused across layers of one staged
        step (the tables do not change between layers).
        """
        self._check_worker()
        if type(layer_index) is not int or not 0 <= layer_index < _LAYERS:
            raise ValueError("layer_index must identify one of the 22 decoder layers")
        request_ids = tuple(request_ids)
        staged = self._staged
        if (
            staged is not None
            and staged.batch is not None
            and staged.batch.requests == request_ids
            and layer_index < staged.written
        ):
            return staged.batch
        handles = np.fromiter(
            (self._handle(r, i + 1) for i, r in enumerate(request_ids)), dtype=np.int64, count=len(request_ids)
        )
        batch = self._upload_batch(request_ids, handles, layer_index)
        if staged is not None and request_ids == staged.requests and layer_index < staged.written:
            staged.batch = batch
        return batch

    def _batch_tables(
        self, request_ids: tuple[RequestId, ...], handles: np.ndarray, layer: int,
        layout: tuple[int, int] | None = None,
    ) -> tuple[np.ndarray, int, kernels.DecodePlan]:
        """Host tables of a batch at ``layer`` in upload order, its block count and plan.

        Order: pieces [grid][4] | row_pieces [B][2] | lengths [B] | prefix [B+1]
        | flat; the pieces come first so the kernel's 16-byte loads of them
        are aligned.  With ``layout=(rows, pieces)`` the first four are padded
        to ``pieces`` pieces and ``rows`` rows: empty pieces (0, 0, 0, 0), rows
        with no pieces (0, 0), length 0 and prefix ``total``, which every
        kernel skips.
        """
        count = len(request_ids)
        if count == 0:
            raise ValueError("attention requires a nonempty batch")
        if layout is not None and count > layout[0]:
            raise ValueError(f"a batch of {count} requests exceeds the layout's {layout[0]} rows")
        host = np.empty(2 * count + 1 + 129 * count, dtype=np.int32)
        try:
            total = self._ledger.batch_into(handles, layer, host)
        except KeyError as error:
            missing = next((r for r in request_ids if r not in self._handles), None)
            raise KeyError(missing) from error
        plan = kernels.decode_plan(self._pool.device, count, total)
        weights = self._slot_weights(plan)
        pieces, row_pieces = kernels.decode_tables(host[count : 2 * count + 1], plan.grid, weights)
        if layout is None:
            tables = np.concatenate((pieces.reshape(-1), row_pieces.reshape(-1), host[: 2 * count + 1 + total]))
            return tables, total, plan
        return padded_tables(pieces, row_pieces, host, count, total, *layout), total, plan

    @staticmethod
    def _device_batch(
        request_ids: tuple[RequestId, ...], tables: np.ndarray, total: int, plan: kernels.DecodePlan, device: Tensor,
        rows: int | None = None, grid: int | None = None,
    ) -> DecodeBatch:
        """A DecodeBatch over ``device``, the uploaded copy of ``tables`` (``rows`` rows, default one per
        request; ``grid`` pieces, default the plan's)."""
        count = len(request_ids) if rows is None else rows
        piece_words = 4 * (plan.grid if grid is None else grid)
        start = piece_words + 2 * count
        return DecodeBatch(
            requests=request_ids,
            pieces=device[:piece_words],
            row_pieces=device[piece_words:start],
            lengths=device[start : start + count],
            prefix=device[start + count : start + 2 * count + 1],
            flat=device[start + 2 * count + 1 : start + 2 * count + 1 + total],
            total_blocks=total,
            plan=plan,
            host_lengths=tables[start : start + count].copy(),
        )

    def _upload_batch(self, request_ids: tuple[RequestId, ...], handles: np.ndarray, layer: int) -> DecodeBatch:
        tables, total, plan = self._batch_tables(request_ids, handles, layer)
        return self._device_batch(request_ids, tables, total, plan, self._upload_i32(tables))

    def _prefill_batch(self, blocks: np.ndarray, start: int, tokens: int) -> DecodeBatch:
        """A prompt chunk as a decode batch: token t is a row of length start + t + 1 over ``blocks``."""
        lengths = np.arange(start + 1, start + tokens + 1, dtype=np.int32)
        counts = -(-lengths // 16)
        prefix = np.concatenate(([0], np.cumsum(counts))).astype(np.int32)
        total = int(prefix[-1])
        flat = blocks[np.arange(total) - np.repeat(prefix[:-1], counts)]
        plan = kernels.decode_plan(self._pool.device, tokens, total)
        pieces, row_pieces = kernels.decode_tables(prefix, plan.grid)
        tables = np.concatenate((pieces.reshape(-1), row_pieces.reshape(-1), lengths, prefix, flat))
        return self._device_batch((), tables, total, plan, self._upload_i32(tables), rows=tokens)

    def attend(self, batch: DecodeBatch, query: Tensor, *, layer_index: int, out: Tensor | None = None) -> Tensor:
        """Decode attention of FP16 query [B, 32, 64] over a :class:`DecodeBatch`."""
        self._check_worker()
        self._window_grid = None  # this launch adds to the slot counters outside a measured window
        if out is None:
            out = torch.empty(query.shape, dtype=torch.float16, device=self._pool.device)
        kernels.decode_attention(
            self._pool,
            layer_index,
            query,
            batch.lengths,
            batch.prefix,
            batch.flat,
            batch.total_blocks,
            batch.plan,
            out,
            self._workspace_for(batch.plan.workspace_bytes),
            self._error,
            batch.pieces,
            batch.row_pieces,
        )
        return out
