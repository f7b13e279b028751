"""ctypes binding of libqkv_sm100.so (declared in include/qkv_sm100.h).

The library is the only compute path of this package: if it is missing or
cannot be loaded, every op raises ``RuntimeError`` — there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_LIB_NAME = "libqkv_sm100.so"
_LIB_PATH = Path(__file__).resolve().parents[1] / _LIB_NAME
_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

QKV_OK = 0
QKV_ERR_INVALID = -1
QKV_ERR_UNSUPPORTED = -2
QKV_ERR_CUDA = -3
QKV_ERR_WORKSPACE = -4
QKV_ERR_DEVICE = -5

QKV_F32, QKV_BF16, QKV_F16 = 0, 1, 2
QKV_I32, QKV_I64 = 0, 1

c_int = ctypes.c_int
c_i64 = ctypes.c_int64
c_size = ctypes.c_size_t
c_float = ctypes.c_float
c_vp = ctypes.c_void_p

# name -> (restype, argtypes); every symbol include/qkv_sm100.h declares
SIGNATURES: dict[str, tuple] = {
    "qkv_version": (ctypes.c_char_p, []),
    "qkv_last_error": (c_int, [ctypes.c_char_p, c_int]),
    "qkv_device_error": (c_int, [ctypes.POINTER(c_int), c_vp]),
    "qkv_int8_scales": (c_int, [c_vp, c_vp, c_i64, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "qkv_int8_quant_store": (
        c_int,
        [c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_int, c_int, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp],
    ),
    "qkv_int8_paged_decode_workspace": (c_size, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "qkv_int8_paged_decode": (
        c_int,
        [
            c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp,
            c_int, c_int, c_int, c_int, c_int, c_i64, c_int, c_float,
            c_vp, c_size, c_vp, c_i64, c_vp,
        ],
    ),
    "qkv_kivi_pack_key": (
        c_int,
        [c_vp, c_int, c_vp, c_int, c_i64, c_int, c_int, c_int, c_int, c_i64, c_vp, c_vp, c_vp, c_vp],
    ),
    "qkv_kivi_pack_kv": (
        c_int,
        [c_vp, c_vp, c_int, c_vp, c_int, c_i64, c_int, c_int, c_int, c_int, c_i64,
         c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
    ),
    "qkv_kivi_pack_value": (
        c_int,
        [c_vp, c_int, c_vp, c_int, c_i64, c_int, c_int, c_int, c_int, c_i64, c_vp, c_vp, c_vp, c_vp],
    ),
    "qkv_kivi_paged_decode_workspace": (c_size, [c_int, c_int, c_int, c_int, c_int, c_int, c_int]),
    "qkv_kivi_paged_decode": (
        c_int,
        [
            c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int,
            c_vp, c_i64, c_vp, c_vp,
            c_int, c_int, c_int, c_int, c_int, c_int, c_i64, c_int, c_float,
            c_vp, c_size, c_vp, c_i64, c_vp,
        ],
    ),
    "qkv_kivi_paged_decode_partials": (
        c_int,
        [
            c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int,
            c_vp, c_i64, c_vp, c_vp,
            c_int, c_int, c_int, c_int, c_int, c_int, c_i64, c_int, c_float,
            c_vp, c_size, c_vp, c_i64, ctypes.POINTER(c_int), c_vp,
        ],
    ),
    "qkv_kivi_paged_decode_noalloc": (
        c_int,
        [
            c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int,
            c_vp, c_i64, c_vp, c_vp,
            c_int, c_int, c_int, c_int, c_int, c_int, c_i64, c_int, c_float,
            c_vp, c_i64, c_vp,
        ],
    ),
    "qkv_dense_prefill_workspace": (c_size, [c_int, c_int, c_int, c_int, c_int]),
    "qkv_dense_prefill": (
        c_int,
        [
            c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_float,
            c_vp, c_size, c_vp, c_vp,
        ],
    ),
    "qkv_kivi_dequant_gather": (
        c_int,
        [
            c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int,
            c_vp, c_i64, c_vp, c_vp, c_vp, c_int,
            c_int, c_int, c_int, c_int, c_i64, c_int, c_vp, c_vp, c_vp,
        ],
    ),
    "qkv_window_create": (c_vp, [c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "qkv_window_destroy": (None, [c_vp]),
    "qkv_window_begin": (None, [c_vp]),
    "qkv_window_store": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_int, c_int]),
    "qkv_window_store_one_each": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int]),
    "qkv_window_flush_direct": (c_int, [c_vp, c_int, c_vp, c_vp, c_int]),
    "qkv_window_prune": (c_int, [c_vp, c_int, c_int, c_vp, c_int]),
    "qkv_window_reset_row": (c_int, [c_vp, c_int]),
    "qkv_window_plan_counts": (c_int, [c_vp, c_int, c_vp, c_vp]),
    "qkv_window_plan_export": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_vp]),
    "qkv_window_expected_live": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_vp]),
    "qkv_kivi_window_gather": (
        c_int, [c_vp, c_vp, c_i64, c_vp, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp],
    ),
    "qkv_kivi_window_scatter": (
        c_int, [c_vp, c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_i64, c_vp, c_i64, c_vp],
    ),
    "qkv_kivi_step_create": (c_vp, []),
    "qkv_kivi_step_destroy": (None, [c_vp]),
    "qkv_kivi_decode_step": (
        c_int,
        [
            c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_int, c_vp, c_i64, c_vp, c_i64, c_vp, c_vp,
            c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
            c_int, c_int, c_int, c_int, c_int, c_i64, c_float, c_vp, c_size, c_vp, c_i64, c_vp,
        ],
    ),
    "qkv_peer_buffer_bytes": (c_size, [c_i64, c_int]),
    "qkv_peer_alloc": (c_int, [c_i64, c_int, ctypes.POINTER(c_vp)]),
    "qkv_peer_free": (c_int, [c_vp]),
    "qkv_ipc_handle": (c_int, [c_vp, c_vp]),
    "qkv_ipc_open": (c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "qkv_ipc_close": (c_int, [c_vp]),
    "qkv_peer_allgather": (c_int, [c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_int, c_int, c_vp]),
    "qkv_peer_combine_allgather": (
        c_int, [c_vp, c_vp, c_int, c_i64, c_int, c_int, c_vp, c_vp, c_i64, c_vp, c_int, c_int, c_vp]),
    "qkv_fp8_store": (
        c_int, [c_vp, c_vp, c_int, c_vp, c_int, c_i64, c_int, c_int, c_int, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp],
    ),
    "qkv_fp8_paged_decode_workspace": (c_size, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "qkv_fp8_paged_decode": (
        c_int,
        [
            c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_int, c_int, c_int, c_int, c_int, c_i64,
            c_int, c_float, c_vp, c_size, c_vp, c_i64, c_vp,
        ],
    ),
    "qkv_fp8_dequant_gather": (
        c_int,
        [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp, c_int, c_int, c_int, c_int, c_i64, c_int, c_vp, c_vp, c_vp],
    ),
    "qkv_int8_dequant_gather": (
        c_int,
        [
            c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp,
            c_int, c_int, c_int, c_int, c_i64, c_int, c_vp, c_vp, c_vp,
        ],
    ),
}


def library_path() -> Path:
    return Path(os.environ.get("QKV_SM100_LIB", str(_LIB_PATH)))


def load() -> ctypes.CDLL:
    """Loads the library once per process and declares every signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"{_LIB_NAME} is not built ({path} is missing); run "
                "`python vllm-ascend-quantized-kv-cache-hust_b200/build.py` "
                "(the quantized-KV kernels have no CPU fallback)"
            )
        try:
            lib = ctypes.CDLL(str(path))
        except OSError as exc:
            raise RuntimeError(f"cannot load {path}: {exc}") from exc
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().qkv_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Raises RuntimeError carrying the library's message when rc != 0."""
    if rc != QKV_OK:
        kind = {
            QKV_ERR_INVALID: "invalid argument",
            QKV_ERR_UNSUPPORTED: "unsupported",
            QKV_ERR_CUDA: "CUDA error",
            QKV_ERR_WORKSPACE: "workspace too small",
            QKV_ERR_DEVICE: "device index error",
        }.get(rc, f"status {rc}")
        raise RuntimeError(f"{what} failed ({kind}): {last_error()}")


def version() -> str:
    return load().qkv_version().decode()


DEVICE_ERRORS = {
    1: "slot out of range",
    2: "block id out of range",
    3: "residual row out of range",
    4: "block table entry negative for a live token",
    5: "a bounded wait on an in-kernel copy gave up",
    6: "window plan source or lane out of range",
    7: "a bounded wait for the other ranks of a peer all-gather gave up",
}


def device_error(stream_handle: int) -> int:
    """Synchronises the stream and returns (and clears) the device error code."""
    code = c_int(0)
    check(load().qkv_device_error(ctypes.byref(code), c_vp(stream_handle)), "qkv_device_error")
    return int(code.value)
