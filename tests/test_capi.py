"""The C ABI surface: the library loads and exports what include/pagedkv.h declares."""

from __future__ import annotations

import ctypes
import re

from pagedcore_b200 import _lib
from tests.conftest import ROOT

HEADER = ROOT / "include" / "pagedkv.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(pkv_[a-z0-9_]+)\s*\(", text))


def test_library_exports_every_declared_symbol() -> None:
    declared = declared_functions()
    assert len(declared) >= 25
    library = ctypes.CDLL(str(_lib.LIBRARY_PATH))
    missing = [name for name in sorted(declared) if not hasattr(library, name)]
    assert missing == []


def test_binding_covers_every_declared_symbol() -> None:
    assert declared_functions() == set(_lib.SIGNATURES)


def test_abi_version_and_error_channel() -> None:
    assert _lib.lib.pkv_abi_version() == 1
    assert _lib.lib.pkv_rope_table_bytes() == 2 * 2048 * 32 * 2
    out = ctypes.c_void_p()
    status = _lib.lib.pkv_ledger_new(0, 1, ctypes.byref(out))
    assert status == _lib.PKV_VALUE_ERROR
    assert b"KV pool must be contiguous" in _lib.lib.pkv_last_error()


def test_device_entry_points_reject_bad_arguments_before_any_launch() -> None:
    # Null pointers are refused on the host: no CUDA call is made.
    status = _lib.lib.pkv_append_kv(None, 1, 0, 1, None, None, 0, 0, None, None, 1, None, None, None, 0, 0, None, None)
    assert status == _lib.PKV_VALUE_ERROR
    status = _lib.lib.pkv_decode_attention(
        None, 1, 0, None, 0, None, None, None, None, None, 1, 1, 1, 1, 1, 1, None, 0, None, 0, None, None
    )
    assert status == _lib.PKV_VALUE_ERROR
    assert b"null pointer" in _lib.lib.pkv_last_error()
    status = _lib.lib.pkv_prefill_attention(None, 1, 0, None, 2048, None, 0, 1, None, 2048, None, None)
    assert status == _lib.PKV_VALUE_ERROR
    assert b"prefill attention: null pointer" in _lib.lib.pkv_last_error()


def test_decode_entry_points_reject_a_partition_that_does_not_cover_the_blocks() -> None:
    # 100 blocks as 10 big pieces of 8 plus tail pieces of 5 need grid 14; grid 12
    # is refused on the host (the pointers are never dereferenced: no launch).
    fake = 1 << 20
    for grid, ok in ((12, False), (15, False), (14, True)):
        status = _lib.lib.pkv_decode_attention(
            fake, 64, 0, fake, 2048, fake, fake, fake, None, None, 4, 100, grid, 8, 10, 5, fake, 2048, None, 0, fake, None
        )
        if ok:
            # The plan passes; the missing workspace is the next thing refused.
            assert status == _lib.PKV_VALUE_ERROR
            assert b"workspace" in _lib.lib.pkv_last_error()
        else:
            assert status == _lib.PKV_VALUE_ERROR
            assert b"launch plan does not match" in _lib.lib.pkv_last_error()


def test_prefill_attention_rejects_bad_arguments_before_any_launch() -> None:
    # Every check below returns before a CUDA call, so none needs a GPU.  The
    # pointers are never dereferenced: each call fails on a size or alignment.
    lib, value_error = _lib.lib, _lib.PKV_VALUE_ERROR
    p = 256  # a nonzero, 16-byte aligned stand-in address
    row = 32 * 64

    def call(layer=0, query=p, query_stride=row, start=0, tokens=1, out=p, out_stride=row, num_blocks=4, pool=p):
        return lib.pkv_prefill_attention(pool, num_blocks, layer, query, query_stride, p, start, tokens, out,
                                         out_stride, p, None)

    for kwargs, message in (
        ({"layer": 22}, b"22 decoder layers"),
        ({"layer": -1}, b"22 decoder layers"),
        ({"tokens": 0}, b"positions below 2048"),
        ({"start": -1}, b"positions below 2048"),
        ({"start": 2040, "tokens": 9}, b"positions below 2048"),
        ({"num_blocks": 0}, b"block count"),
        ({"query": p + 2}, b"misaligned"),
        ({"query_stride": row - 2}, b"misaligned"),
        ({"out_stride": row + 1}, b"misaligned"),
        ({"pool": p + 8}, b"misaligned"),
    ):
        assert call(**kwargs) == value_error, kwargs
        assert message in lib.pkv_last_error(), (kwargs, lib.pkv_last_error())
