"""ctypes binding of ``libpagedkv.so`` (the C ABI of ``include/pagedkv.h``).

The library is built in-tree by :mod:`pagedcore_b200.build`.  Importing this
module loads it; a missing library raises immediately, because every device
operation of this package goes through it and there is no fallback path.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_void_p
from pathlib import Path

from pagedcore_b200 import build as _build

PKV_OK = 0
PKV_VALUE_ERROR = 1
PKV_RUNTIME_ERROR = 2
PKV_KEY_ERROR = 3
PKV_CUDA_ERROR = 4

VALIDATE_INCREMENTAL = 0
VALIDATE_FULL = 1
VIEW_STAGED = -2

DEVICE_BAD_BLOCK = 1
DEVICE_BAD_POSITION = 2
DEVICE_WAIT_TIMEOUT = 4

DECODE_EARLY_KV = 1

LIBRARY_PATH: Path = _build.LIBRARY

i32p = POINTER(c_int32)
i64p = POINTER(c_int64)

# name -> (restype, argtypes); every symbol declared in include/pagedkv.h.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "pkv_last_error": (c_char_p, []),
    "pkv_abi_version": (c_int, []),
    "pkv_ledger_new": (c_int, [c_int32, c_int32, POINTER(c_void_p)]),
    "pkv_ledger_free": (None, [c_void_p]),
    "pkv_ledger_set_validation": (c_int, [c_void_p, c_int32]),
    "pkv_ledger_reserve": (c_int, [c_void_p, c_int64, c_int64]),
    "pkv_ledger_release": (c_int, [c_void_p, c_int64]),
    "pkv_ledger_capacity": (c_int, [c_void_p, i64p]),
    "pkv_ledger_length": (c_int, [c_void_p, c_int64, i32p]),
    "pkv_ledger_table": (c_int, [c_void_p, c_int64, i32p, c_int32, i32p]),
    "pkv_ledger_append_plan": (c_int, [c_void_p, c_int64, c_int32, c_void_p, i32p]),
    "pkv_ledger_append_commit": (c_int, [c_void_p, c_int64, c_int32]),
    "pkv_ledger_append_plan_many": (c_int, [c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_void_p]),
    "pkv_ledger_append_commit_many": (c_int, [c_void_p, c_void_p, c_void_p, c_int32]),
    "pkv_ledger_decode_begin": (c_int, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p]),
    "pkv_ledger_decode_check": (c_int, [c_void_p, c_int64, c_int32, i32p, i32p]),
    "pkv_ledger_decode_mark": (c_int, [c_void_p, c_int64, c_int32]),
    "pkv_ledger_decode_mark_layers": (c_int, [c_void_p, c_int32, c_int32]),
    "pkv_ledger_decode_commit": (c_int, [c_void_p]),
    "pkv_ledger_decode_abort": (None, [c_void_p]),
    "pkv_ledger_decode_active": (c_int, [c_void_p]),
    "pkv_ledger_view": (c_int, [c_void_p, c_int64, c_int32, i32p, c_int32, i32p, i32p]),
    "pkv_ledger_batch": (
        c_int,
        [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_int32, i32p],
    ),
    "pkv_ledger_audit": (c_int, [c_void_p]),
    "pkv_ledger_free_list": (c_int, [c_void_p, i32p, c_int32, i32p]),
    "pkv_ledger_reorder_free": (c_int, [c_void_p, i32p, c_int32]),
    "pkv_ledger_debug_set_table": (c_int, [c_void_p, c_int64, i32p, c_int32, c_int32]),
    "pkv_ledger_debug_set_free": (c_int, [c_void_p, i32p, c_int32]),
    "pkv_rope_table_bytes": (c_int64, []),
    "pkv_add_rms_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_float, c_void_p]),
    "pkv_silu_mul": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_void_p]),
    "pkv_gemv": (c_int, [c_void_p, c_int64, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p]),
    "pkv_linear_splits": (c_int, [c_int32, c_int32, c_int32, i32p]),
    "pkv_linear": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_void_p,
         c_void_p],
    ),
    "pkv_split_sum": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p]),
    "pkv_add_rms_norm_split": (
        c_int, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_float, c_void_p],
    ),
    "pkv_silu_mul_split": (c_int, [c_void_p, c_int32, c_void_p, c_int32, c_int32, c_void_p]),
    "pkv_append_kv": (
        c_int,
        [
            c_void_p,
            c_int32,
            c_int32,
            c_int32,
            c_void_p,
            c_void_p,
            c_int64,
            c_int64,
            c_void_p,
            c_void_p,
            c_int32,
            c_void_p,
            c_void_p,
            c_void_p,
            c_int64,
            c_int64,
            c_void_p,
            c_void_p,
        ],
    ),
    "pkv_decode_plan": (c_int, [c_int32, c_int32, c_int32, i32p, i32p, i32p, i32p, i64p]),
    "pkv_decode_tables": (c_int, [c_void_p, c_int32, c_int32, c_void_p, ctypes.c_float, c_void_p, c_void_p]),
    "pkv_decode_layer": (
        c_int,
        [
            c_void_p,  # pool
            c_int32,  # num_blocks
            c_int32,  # layer
            c_void_p,  # query
            c_int64,  # query_stride
            c_void_p,  # key
            c_void_p,  # value
            c_int64,  # kv_stride
            c_void_p,  # rope_table
            c_void_p,  # lengths
            c_void_p,  # prefix
            c_void_p,  # flat
            c_void_p,  # pieces
            c_void_p,  # row_pieces
            c_int32,  # batch
            c_int32,  # total_blocks
            c_int32,  # grid
            c_int32,  # blocks_per_cta
            c_int32,  # big_ctas
            c_int32,  # tail_blocks
            c_void_p,  # out
            c_int64,  # out_stride
            c_void_p,  # workspace
            c_int64,  # workspace_bytes
            c_void_p,  # error_flag
            c_int32,  # flags
            c_void_p,  # stream
        ],
    ),
    "pkv_decode_attention_noalloc": (
        c_int,
        [
            c_void_p,  # pool
            c_int32,  # num_blocks
            c_int32,  # layer
            c_void_p,  # query
            c_int64,  # query_stride
            c_void_p,  # lengths
            c_void_p,  # prefix
            c_void_p,  # flat
            c_void_p,  # pieces
            c_void_p,  # row_pieces
            c_int32,  # batch
            c_int32,  # total_blocks
            c_int32,  # grid
            c_int32,  # blocks_per_cta
            c_int32,  # big_ctas
            c_int32,  # tail_blocks
            c_void_p,  # out
            c_int64,  # out_stride
            c_void_p,  # error_flag
            c_void_p,  # stream
        ],
    ),
    "pkv_decode_attention": (
        c_int,
        [
            c_void_p,  # pool
            c_int32,  # num_blocks
            c_int32,  # layer
            c_void_p,  # query
            c_int64,  # query_stride
            c_void_p,  # lengths
            c_void_p,  # prefix
            c_void_p,  # flat
            c_void_p,  # pieces
            c_void_p,  # row_pieces
            c_int32,  # batch
            c_int32,  # total_blocks
            c_int32,  # grid
            c_int32,  # blocks_per_cta
            c_int32,  # big_ctas
            c_int32,  # tail_blocks
            c_void_p,  # out
            c_int64,  # out_stride
            c_void_p,  # workspace
            c_int64,  # workspace_bytes
            c_void_p,  # error_flag
            c_void_p,  # stream
        ],
    ),
    "pkv_prefill_attention": (
        c_int,
        [
            c_void_p,  # pool
            c_int32,  # num_blocks
            c_int32,  # layer
            c_void_p,  # query
            c_int64,  # query_stride
            c_void_p,  # blocks
            c_int32,  # start
            c_int32,  # tokens
            c_void_p,  # out
            c_int64,  # out_stride
            c_void_p,  # error_flag
            c_void_p,  # stream
        ],
    ),
}


def _load() -> ctypes.CDLL:
    if not LIBRARY_PATH.exists():
        raise ImportError(
            f"{LIBRARY_PATH} is missing: build it with `python -m pagedcore_b200.build` "
            "(the paged KV path has no non-native fallback)"
        )
    library = ctypes.CDLL(str(LIBRARY_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        function = getattr(library, name)
        function.restype = restype
        function.argtypes = argtypes
    return library


lib = _load()

_EXCEPTIONS: dict[int, type[Exception]] = {
    PKV_VALUE_ERROR: ValueError,
    PKV_RUNTIME_ERROR: RuntimeError,
    PKV_KEY_ERROR: KeyError,
    PKV_CUDA_ERROR: RuntimeError,
}


def error_for(status: int) -> Exception:
    message = (lib.pkv_last_error() or b"").decode("utf-8", "replace")
    return _EXCEPTIONS.get(status, RuntimeError)(message or f"libpagedkv status {status}")


def check(status: int) -> None:
    """Raise the exception class the reference raises for this status."""
    if status != PKV_OK:
        raise error_for(status)


def device_error_message(flag: int) -> str:
    parts = []
    if flag & DEVICE_BAD_BLOCK:
        parts.append("physical KV block outside the pool")
    if flag & DEVICE_BAD_POSITION:
        parts.append("RoPE position outside [0, 2048)")
    if flag & DEVICE_WAIT_TIMEOUT:
        parts.append("a bounded pipeline wait timed out")
    return "KV kernel reported: " + ", ".join(parts or [f"flag {flag}"])
