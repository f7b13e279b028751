"""The C-ABI library loads and exports every symbol include/qkv_sm100.h
declares; argument errors come back as status codes with messages, before any
device work (so these run without a GPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from qkv_b200.ops import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "qkv_sm100.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^QKV_API\s+[\w\s\*]+?\b(qkv_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_abi():
    names = declared_symbols()
    assert {"qkv_version", "qkv_last_error", "qkv_kivi_pack_key", "qkv_kivi_paged_decode"} <= names


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(_lib.SIGNATURES) == declared_symbols()
    assert "sm_100a" in _lib.version()


def test_invalid_arguments_return_status_and_message():
    lib = _lib.load()
    rc = lib.qkv_kivi_pack_key(None, 1, None, 1, 16, 2, 32, 7, 16, 4, None, None, None, None)
    assert rc == _lib.QKV_ERR_INVALID
    assert "group_size" in _lib.last_error()
    rc = lib.qkv_kivi_pack_value(None, 9, None, 1, 16, 2, 32, 8, 16, 4, None, None, None, None)
    assert rc == _lib.QKV_ERR_INVALID and "dtype" in _lib.last_error()
    rc = lib.qkv_kivi_paged_decode(
        None, 0, None, None, None, None, None, None, None, None, 0, 0, None, 0, None, None,
        1, 30, 8, 128, 128, 128, 4, 100, 0.1, None, 0, None, 0, None,
    )
    assert rc == _lib.QKV_ERR_INVALID and "num_heads" in _lib.last_error()
    with pytest.raises(RuntimeError, match="invalid argument"):
        _lib.check(rc, "qkv_kivi_paged_decode")


def test_zero_sized_calls_are_no_ops():
    lib = _lib.load()
    assert lib.qkv_kivi_pack_key(None, 1, None, 1, 0, 2, 32, 8, 16, 4, None, None, None, None) == 0
    assert lib.qkv_int8_quant_store(None, None, None, 1, 0, 8, 128, 128, 4, None, None, None, None, None) == 0


def test_workspace_queries_are_pure():
    lib = _lib.load()
    assert lib.qkv_kivi_paged_decode_workspace(8, 40, 8, 128, 128, 128, 8192) > 0
    assert lib.qkv_int8_paged_decode_workspace(0, 32, 8, 128, 128, 8192) == 0


def test_ops_refuse_cpu_tensors():
    import torch

    from qkv_b200.ops import kivi_pack_value_cache

    v = torch.zeros(2, 2, 32)
    views = (torch.zeros(4, 16, 2, 4, dtype=torch.int32), torch.zeros(4, 16, 2, 4), torch.zeros(4, 16, 2, 4))
    with pytest.raises(RuntimeError, match="needs CUDA"):
        kivi_pack_value_cache(v, torch.arange(2), *views, 8)


def test_peer_allgather_sizes_and_argument_checks():
    """The NVLink peer all-gather entry points validate before touching the
    device: bad world / rank, row sizes, slices larger than the buffers and
    null pointers come back as QKV_ERR_INVALID with a message."""
    import ctypes

    lib = _lib.load()
    # receive words: 2 parities x world x (slice / 4) words x 8 bytes, plus 64 control bytes
    assert lib.qkv_peer_buffer_bytes(65536, 8) == 2 * 8 * (65536 // 4) * 8 + 64
    assert lib.qkv_peer_buffer_bytes(0, 8) == 0
    bufs = (ctypes.c_void_p * 2)(16, 32)
    addr = ctypes.addressof(bufs)
    cases = [
        ((16, 4, 64, addr, 4096, 16, 0, 9, None), "world must be 1..8"),
        ((16, 4, 64, addr, 4096, 16, 2, 2, None), "rank inside it"),
        ((16, 4, 62, addr, 4096, 16, 0, 2, None), "multiple of 4 bytes"),
        ((16, 100, 64, addr, 4096, 16, 0, 2, None), "does not fit"),
        ((None, 4, 64, addr, 4096, 16, 0, 2, None), "null pointer"),
        ((18, 4, 64, addr, 4096, 16, 0, 2, None), "4-byte aligned"),
    ]
    for args, match in cases:
        assert lib.qkv_peer_allgather(*args) == _lib.QKV_ERR_INVALID
        assert match in _lib.last_error(), (args, _lib.last_error())
    # the combine + gather checks its own arguments the same way
    rc = lib.qkv_peer_combine_allgather(16, 32, 4, 4, 0, 128, 16, addr, 4096, 16, 0, 2, None)
    assert rc == _lib.QKV_ERR_INVALID and "head sizes" in _lib.last_error()
    rc = lib.qkv_peer_combine_allgather(None, 32, 4, 4, 2, 128, 16, addr, 1 << 20, 16, 0, 2, None)
    assert rc == _lib.QKV_ERR_INVALID and "null pointer" in _lib.last_error()
    out = ctypes.c_void_p()
    assert lib.qkv_peer_alloc(10, 2, ctypes.byref(out)) == _lib.QKV_ERR_INVALID  # not a multiple of 16
    assert lib.qkv_ipc_handle(None, None) == _lib.QKV_ERR_INVALID
