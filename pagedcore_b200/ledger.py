"""Python view of the C++ block ledger (``pkv_ledger_*`` in include/pagedkv.h).

``BlockLedger`` holds the whole bookkeeping of the paged KV cache - LIFO free
stack, per-request credits, tables and lengths, staged decode - with integer
request handles.  :class:`pagedcore_b200.kv_cache.KVAllocator` composes it
with the device pool; it is also usable on its own (it needs no GPU), which is
how the bookkeeping is tested against the oracle on CPU.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence

import numpy as np

from pagedcore_b200._lib import VALIDATE_FULL, VALIDATE_INCREMENTAL, check, lib

_VALIDATION = {"full": VALIDATE_FULL, "incremental": VALIDATE_INCREMENTAL}
_MAX_TABLE = 129  # 128 credits + one staged block


def _i32(array: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(array.ctypes.data)


class BlockLedger:
    """Block assignment state for one pool of ``num_blocks`` blocks."""

    def __init__(self, num_blocks: int, validation: str = "full") -> None:
        if validation not in _VALIDATION:
            raise ValueError(f"validation must be one of {sorted(_VALIDATION)}")
        handle = ctypes.c_void_p()
        check(lib.pkv_ledger_new(int(num_blocks), _VALIDATION[validation], ctypes.byref(handle)))
        self._handle = handle
        self.num_blocks = int(num_blocks)

    def __del__(self) -> None:
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            lib.pkv_ledger_free(handle)
            self._handle = None

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._handle

    def set_validation(self, validation: str) -> None:
        check(lib.pkv_ledger_set_validation(self._handle, _VALIDATION[validation]))

    # -- requests -----------------------------------------------------------
    def reserve(self, request: int, credits: int) -> None:
        check(lib.pkv_ledger_reserve(self._handle, request, credits))

    def release(self, request: int) -> None:
        check(lib.pkv_ledger_release(self._handle, request))

    def capacity(self) -> tuple[int, int, int, int, int, int]:
        out = (ctypes.c_int64 * 6)()
        check(lib.pkv_ledger_capacity(self._handle, out))
        return tuple(int(v) for v in out)  # type: ignore[return-value]

    def length(self, request: int) -> int:
        out = ctypes.c_int32()
        check(lib.pkv_ledger_length(self._handle, request, ctypes.byref(out)))
        return out.value

    def table(self, request: int) -> tuple[int, ...]:
        buffer = (ctypes.c_int32 * _MAX_TABLE)()
        count = ctypes.c_int32()
        check(lib.pkv_ledger_table(self._handle, request, buffer, _MAX_TABLE, ctypes.byref(count)))
        return tuple(buffer[: count.value])

    # -- prompt append ------------------------------------------------------
    def append_plan(self, request: int, tokens: int) -> tuple[np.ndarray, int]:
        """Slot ids of the next ``tokens`` positions and the first position."""
        slots = np.empty(max(int(tokens), 1), dtype=np.int32)
        start = ctypes.c_int32()
        check(lib.pkv_ledger_append_plan(self._handle, request, int(tokens), _i32(slots), ctypes.byref(start)))
        return slots[: int(tokens)], start.value

    def append_commit(self, request: int, tokens: int) -> None:
        check(lib.pkv_ledger_append_commit(self._handle, request, int(tokens)))

    def append(self, request: int, tokens: int) -> np.ndarray:
        slots, _ = self.append_plan(request, tokens)
        self.append_commit(request, tokens)
        return slots

    def append_plan_many(self, requests: Sequence[int], tokens: Sequence[int]) -> tuple[np.ndarray, np.ndarray]:
        """Slot ids of several appends planned in order (request i as if 0..i-1 were committed).

        Returns the slots of all requests concatenated and each request's first position.
        """
        handles = np.ascontiguousarray(requests, dtype=np.int64)
        counts = np.ascontiguousarray(tokens, dtype=np.int32)
        if handles.shape != counts.shape or handles.ndim != 1:
            raise ValueError("requests and tokens must be two sequences of one length")
        slots = np.empty(max(int(counts.sum()), 1), dtype=np.int32)
        starts = np.empty(max(len(handles), 1), dtype=np.int32)
        check(lib.pkv_ledger_append_plan_many(self._handle, handles.ctypes.data, counts.ctypes.data, len(handles),
                                              _i32(slots), _i32(starts)))
        return slots[: int(counts.sum())], starts[: len(handles)]

    def append_commit_many(self, requests: Sequence[int], tokens: Sequence[int]) -> None:
        handles = np.ascontiguousarray(requests, dtype=np.int64)
        counts = np.ascontiguousarray(tokens, dtype=np.int32)
        if handles.shape != counts.shape or handles.ndim != 1:
            raise ValueError("requests and tokens must be two sequences of one length")
        check(lib.pkv_ledger_append_commit_many(self._handle, handles.ctypes.data, counts.ctypes.data, len(handles)))

    # -- staged one-token decode -------------------------------------------
    def decode_begin(self, requests: Sequence[int]) -> tuple[np.ndarray, np.ndarray]:
        handles = np.asarray(requests, dtype=np.int64)
        count = len(handles)
        slots = np.empty(max(count, 1), dtype=np.int32)
        positions = np.empty(max(count, 1), dtype=np.int32)
        check(
            lib.pkv_ledger_decode_begin(
                self._handle, ctypes.c_void_p(handles.ctypes.data), count, _i32(slots), _i32(positions)
            )
        )
        return slots[:count], positions[:count]

    def decode_check(self, request: int, layer: int) -> tuple[int, int]:
        slot = ctypes.c_int32()
        position = ctypes.c_int32()
        check(lib.pkv_ledger_decode_check(self._handle, request, layer, ctypes.byref(slot), ctypes.byref(position)))
        return slot.value, position.value

    def decode_mark(self, request: int, layer: int) -> None:
        check(lib.pkv_ledger_decode_mark(self._handle, request, layer))

    def decode_mark_layers(self, first: int, count: int) -> None:
        """Record layers first..first+count-1 written for every staged row."""
        check(lib.pkv_ledger_decode_mark_layers(self._handle, first, count))

    def decode_commit(self) -> None:
        check(lib.pkv_ledger_decode_commit(self._handle))

    def decode_abort(self) -> None:
        lib.pkv_ledger_decode_abort(self._handle)

    @property
    def staging(self) -> bool:
        return bool(lib.pkv_ledger_decode_active(self._handle))

    # -- reader views ---------------------------------------------------------
    def view(self, request: int, layer: int) -> tuple[tuple[int, ...], int]:
        buffer = (ctypes.c_int32 * _MAX_TABLE)()
        count = ctypes.c_int32()
        length = ctypes.c_int32()
        check(
            lib.pkv_ledger_view(
                self._handle, request, layer, buffer, _MAX_TABLE, ctypes.byref(count), ctypes.byref(length)
            )
        )
        return tuple(buffer[: count.value]), length.value

    def batch_into(self, requests: np.ndarray, layer: int, out: np.ndarray) -> int:
        """Write lengths[B] | prefix[B+1] | flat tables into ``out``; return total blocks."""
        count = len(requests)
        total = ctypes.c_int32()
        base = out.ctypes.data
        check(
            lib.pkv_ledger_batch(
                self._handle,
                ctypes.c_void_p(requests.ctypes.data),
                count,
                layer,
                ctypes.c_void_p(base),
                ctypes.c_void_p(base + 4 * count),
                ctypes.c_void_p(base + 4 * (2 * count + 1)),
                len(out) - (2 * count + 1),
                ctypes.byref(total),
            )
        )
        return total.value

    def batch(self, requests: Sequence[int], layer: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        handles = np.asarray(requests, dtype=np.int64)
        count = len(handles)
        out = np.empty(2 * count + 1 + _MAX_TABLE * count, dtype=np.int32)
        total = self.batch_into(handles, layer, out)
        return out[:count].copy(), out[count : 2 * count + 1].copy(), out[2 * count + 1 : 2 * count + 1 + total].copy()

    # -- invariants and white-box access --------------------------------------
    def audit(self) -> None:
        check(lib.pkv_ledger_audit(self._handle))

    def free_list(self) -> list[int]:
        buffer = np.empty(self.num_blocks + 1, dtype=np.int32)
        count = ctypes.c_int32()
        check(
            lib.pkv_ledger_free_list(
                self._handle, buffer.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(buffer), ctypes.byref(count)
            )
        )
        return buffer[: count.value].tolist()

    def reorder_free(self, blocks: Sequence[int]) -> None:
        array = np.asarray(blocks, dtype=np.int32)
        check(
            lib.pkv_ledger_reorder_free(
                self._handle, array.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(array)
            )
        )

    def debug_set_table(self, request: int, blocks: Sequence[int], length: int) -> None:
        array = np.asarray(blocks, dtype=np.int32)
        check(
            lib.pkv_ledger_debug_set_table(
                self._handle, request, array.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(array), length
            )
        )

    def debug_set_free(self, blocks: Sequence[int]) -> None:
        array = np.asarray(blocks, dtype=np.int32)
        check(
            lib.pkv_ledger_debug_set_free(
                self._handle, array.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(array)
            )
        )
