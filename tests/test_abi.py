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
