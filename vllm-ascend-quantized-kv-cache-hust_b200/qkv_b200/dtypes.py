"""Quantized-KV dtype literal -> quantisation mode -> storage layout.

The contract of the reference's layer 0 (dtypes.py:15-94 of
vllm_ascend_quantized_kv_cache): the CLI literals this package serves,
``int8``, ``kivi_int4`` and ``fp8_per_token_head``, and fail-closed resolution
of everything else.
Pure Python, importable anywhere.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import IntEnum


class KVQuantMode(IntEnum):
    """Quantisation modes; values match the reference's enum (dtypes.py:15-22)."""

    NONE = 0
    INT8_PER_TENSOR = 8
    KIVI_INT4 = 9
    FP8_PER_TOKEN_HEAD = 10


def get_kv_quant_mode(dtype: str) -> KVQuantMode:
    """``int8`` / ``kivi_int4`` / ``fp8_per_token_head`` -> their mode; any
    other literal -> NONE."""
    return {
        "int8": KVQuantMode.INT8_PER_TENSOR,
        "kivi_int4": KVQuantMode.KIVI_INT4,
        "fp8_per_token_head": KVQuantMode.FP8_PER_TOKEN_HEAD,
    }.get(dtype, KVQuantMode.NONE)


def is_quantized_kv_cache(dtype: str) -> bool:
    return get_kv_quant_mode(dtype) is not KVQuantMode.NONE


def int4_packed_dim(head_size: int) -> int:
    """Bytes per head row of int4 codes: two lanes per byte."""
    if head_size <= 0 or head_size % 2:
        raise ValueError("INT4 head_size must be a positive even number")
    return head_size // 2


@dataclass(frozen=True)
class KVCacheLayout:
    """Resolved storage layout of one cache dtype literal."""

    dtype: str
    head_size: int
    storage_dtype: str
    packed_last_dim: int
    quant_mode: KVQuantMode


def resolve_layout(dtype: str, head_size: int) -> KVCacheLayout:
    """``int8``: int8 storage, last dim = head_size; ``kivi_int4``: uint8,
    head_size / 2; ``fp8_per_token_head``: uint8 E4M3 bytes, head_size (a
    multiple of 4; the fp32 scales are budgeted by the method's byte layout);
    anything else raises ValueError."""
    mode = get_kv_quant_mode(dtype)
    if mode is KVQuantMode.INT8_PER_TENSOR:
        if head_size <= 0:
            raise ValueError("head_size must be positive")
        return KVCacheLayout(dtype, head_size, "int8", head_size, mode)
    if mode is KVQuantMode.KIVI_INT4:
        return KVCacheLayout(dtype, head_size, "uint8", int4_packed_dim(head_size), mode)
    if mode is KVQuantMode.FP8_PER_TOKEN_HEAD:
        if head_size <= 0 or head_size % 4:
            raise ValueError(
                "fp8_per_token_head requires head_size positive and divisible "
                f"by 4 (fp32 scale alignment), got {head_size}"
            )
        return KVCacheLayout(dtype, head_size, "uint8", head_size, mode)
    raise ValueError(f"dtype is not a registered quantized KV layout: {dtype}")


__all__ = [
    "KVCacheLayout",
    "KVQuantMode",
    "get_kv_quant_mode",
    "int4_packed_dim",
    "is_quantized_kv_cache",
    "resolve_layout",
]
