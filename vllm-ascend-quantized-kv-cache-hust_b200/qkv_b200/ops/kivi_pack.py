"""KIVI INT4 pack ops on B200 — drop-in for the reference's triton pack entry
points (ops/triton/kivi_pack.py:229-348): same names, arguments, validators and
error messages; the work runs in qkv_kivi_pack_key / qkv_kivi_pack_value of
libqkv_sm100.so on the current CUDA stream."""

from __future__ import annotations

import torch

from . import _lib
from ._torch import dtype_code, index_code, ptr, require_cuda, stream_handle
from .kivi_layout import (
    _check_contiguous,
    _check_key_cache_layout,
    _check_key_slot_groups,
    _check_same_device,
    _check_slot_mapping,
    _check_value_cache_layout,
)


def kivi_pack_value_cache(
    value: torch.Tensor,
    slot_mapping: torch.Tensor,
    v_quant_cache: torch.Tensor,
    v_scale_cache: torch.Tensor,
    v_mn_cache: torch.Tensor,
    group_size: int,
) -> None:
    """Packs values ``[num_tokens, KVH, D]`` (fp32/bf16/fp16) into the paged int4
    value view, one token per slot, grouped along the head dimension."""
    num_tokens, num_kv_heads, head_size = value.shape
    if num_tokens == 0:
        return
    assert group_size % 8 == 0
    assert head_size % group_size == 0
    assert head_size % 8 == 0
    for name, t in (
        ("value", value),
        ("slot_mapping", slot_mapping),
        ("v_quant_cache", v_quant_cache),
        ("v_scale_cache", v_scale_cache),
        ("v_mn_cache", v_mn_cache),
    ):
        _check_contiguous(name, t)
    for name, t in (
        ("slot_mapping", slot_mapping),
        ("v_quant_cache", v_quant_cache),
        ("v_scale_cache", v_scale_cache),
        ("v_mn_cache", v_mn_cache),
    ):
        _check_same_device(name, t, value)
    _check_slot_mapping(slot_mapping, num_tokens)
    _check_value_cache_layout(
        v_quant_cache, v_scale_cache, v_mn_cache,
        num_kv_heads=num_kv_heads, head_size=head_size, group_size=group_size,
    )
    require_cuda("kivi_pack_value_cache", value)
    nb, block = v_quant_cache.shape[:2]
    lib = _lib.load()
    rc = lib.qkv_kivi_pack_value(
        ptr(value), dtype_code(value), ptr(slot_mapping), index_code(slot_mapping),
        num_tokens, num_kv_heads, head_size, group_size, block, nb,
        ptr(v_quant_cache), ptr(v_scale_cache), ptr(v_mn_cache), stream_handle(value.device),
    )
    _lib.check(rc, "kivi_pack_value_cache")


def kivi_pack_key_cache(
    key: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_quant_cache: torch.Tensor,
    k_scale_cache: torch.Tensor,
    k_mn_cache: torch.Tensor,
    group_size: int,
    *,
    validate_slots: bool = True,
) -> None:
    """Packs whole token groups of keys ``[n*g, KVH, D]`` into the paged int4
    key view (8 tokens of one channel per int32 word).

    ``validate_slots=False`` skips the value-level slot-group gate when the
    caller has already proven alignment on host (the residual-window flush
    does), saving the device->host reads the gate needs."""
    num_tokens, num_kv_heads, head_size = key.shape
    if num_tokens == 0:
        return
    assert group_size % 8 == 0
    assert num_tokens % group_size == 0
    assert head_size % 8 == 0
    for name, t in (
        ("key", key),
        ("slot_mapping", slot_mapping),
        ("k_quant_cache", k_quant_cache),
        ("k_scale_cache", k_scale_cache),
        ("k_mn_cache", k_mn_cache),
    ):
        _check_contiguous(name, t)
    for name, t in (
        ("slot_mapping", slot_mapping),
        ("k_quant_cache", k_quant_cache),
        ("k_scale_cache", k_scale_cache),
        ("k_mn_cache", k_mn_cache),
    ):
        _check_same_device(name, t, key)
    _check_slot_mapping(slot_mapping, num_tokens)
    block_size = _check_key_cache_layout(
        k_quant_cache, k_scale_cache, k_mn_cache,
        num_kv_heads=num_kv_heads, head_size=head_size, group_size=group_size,
    )
    if validate_slots:
        _check_key_slot_groups(slot_mapping, block_size=block_size, group_size=group_size)
    require_cuda("kivi_pack_key_cache", key)
    lib = _lib.load()
    rc = lib.qkv_kivi_pack_key(
        ptr(key), dtype_code(key), ptr(slot_mapping), index_code(slot_mapping),
        num_tokens, num_kv_heads, head_size, group_size, block_size, k_quant_cache.shape[0],
        ptr(k_quant_cache), ptr(k_scale_cache), ptr(k_mn_cache), stream_handle(key.device),
    )
    _lib.check(rc, "kivi_pack_key_cache")


def kivi_pack_kv_cache(
    key: torch.Tensor,
    value: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_caches: tuple,
    v_caches: tuple,
    group_size: int,
    *,
    validate_slots: bool = True,
) -> None:
    """``kivi_pack_key_cache(key, ...)`` then ``kivi_pack_value_cache(value,
    ...)`` on the same slots, as one launch (``qkv_kivi_pack_kv``): the bulk
    prompt write's flush of both sides. ``k_caches`` = (k_quant, k_scale,
    k_mn), ``v_caches`` = (v_quant, v_scale, v_mn); the same validators and
    messages as the two calls."""
    num_tokens, num_kv_heads, head_size = key.shape
    if num_tokens == 0:
        return
    if value.shape != key.shape or value.dtype != key.dtype:
        raise RuntimeError("kivi_pack_kv_cache: key and value must have the same shape and dtype.")
    assert group_size % 8 == 0
    assert num_tokens % group_size == 0
    assert head_size % group_size == 0
    assert head_size % 8 == 0
    k_quant, k_scale, k_mn = k_caches
    v_quant, v_scale, v_mn = v_caches
    for name, t in (("key", key), ("value", value), ("slot_mapping", slot_mapping), ("k_quant_cache", k_quant),
                    ("k_scale_cache", k_scale), ("k_mn_cache", k_mn), ("v_quant_cache", v_quant),
                    ("v_scale_cache", v_scale), ("v_mn_cache", v_mn)):
        _check_contiguous(name, t)
    for name, t in (("value", value), ("slot_mapping", slot_mapping), ("k_quant_cache", k_quant),
                    ("k_scale_cache", k_scale), ("k_mn_cache", k_mn), ("v_quant_cache", v_quant),
                    ("v_scale_cache", v_scale), ("v_mn_cache", v_mn)):
        _check_same_device(name, t, key)
    _check_slot_mapping(slot_mapping, num_tokens)
    block_size = _check_key_cache_layout(
        k_quant, k_scale, k_mn, num_kv_heads=num_kv_heads, head_size=head_size, group_size=group_size,
    )
    _check_value_cache_layout(
        v_quant, v_scale, v_mn, num_kv_heads=num_kv_heads, head_size=head_size, group_size=group_size,
    )
    if validate_slots:
        _check_key_slot_groups(slot_mapping, block_size=block_size, group_size=group_size)
    require_cuda("kivi_pack_kv_cache", key, value)
    lib = _lib.load()
    rc = lib.qkv_kivi_pack_kv(
        ptr(key), ptr(value), dtype_code(key), ptr(slot_mapping), index_code(slot_mapping),
        num_tokens, num_kv_heads, head_size, group_size, block_size, k_quant.shape[0],
        ptr(k_quant), ptr(k_scale), ptr(k_mn), ptr(v_quant), ptr(v_scale), ptr(v_mn), stream_handle(key.device),
    )
    _lib.check(rc, "kivi_pack_kv_cache")


__all__ = ["kivi_pack_key_cache", "kivi_pack_kv_cache", "kivi_pack_value_cache"]
