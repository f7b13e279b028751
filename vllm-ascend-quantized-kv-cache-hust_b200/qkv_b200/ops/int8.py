"""INT8 dynamic per-channel ops on B200: scale calibration, quantised paged
write and paged decode attention (libqkv_sm100.so)."""

from __future__ import annotations

import torch

from . import _lib
from ._torch import WORKSPACE, index_code, ptr, require_cuda, stream_handle


def int8_calc_scales(key: torch.Tensor, value: torch.Tensor):
    """Scales of ``_prepare_int8_scales`` (methods/int8_dynamic/
    attention_backend.py:130-150) from bf16 ``[T, KVH, D]`` K/V.

    Returns ``(k_inv, v_inv, k_aq, v_aq)``, bf16 ``[KVH, D]`` each."""
    require_cuda("int8_calc_scales", key, value)
    if key.dtype != torch.bfloat16 or value.dtype != torch.bfloat16:
        raise RuntimeError("int8_calc_scales expects bfloat16 key/value")
    key = key.contiguous()
    value = value.contiguous()
    T, H, D = key.shape
    out = [torch.empty(H, D, dtype=torch.bfloat16, device=key.device) for _ in range(4)]
    rc = _lib.load().qkv_int8_scales(
        ptr(key), ptr(value), T, H, D, *(ptr(t) for t in out), stream_handle(key.device)
    )
    _lib.check(rc, "int8_calc_scales")
    return tuple(out)


def int8_quant_store(key, value, slot_mapping, k_inv, v_inv, key_cache, value_cache) -> None:
    """Quantise bf16 K/V ``[T, KVH, D]`` and scatter them into int8 pages
    ``[NB, blk, KVH, D]`` (``_quantize_kv_to_runtime_int8`` + the host's
    reshape_and_cache, attention_backend.py:82-88)."""
    require_cuda("int8_quant_store", key, value, key_cache, value_cache)
    T, H, D = key.shape
    if T == 0:
        return
    key = key.contiguous()
    value = value.contiguous()
    slot_mapping = slot_mapping.contiguous()
    nb, blk = key_cache.shape[:2]
    rc = _lib.load().qkv_int8_quant_store(
        ptr(key), ptr(value), ptr(slot_mapping), index_code(slot_mapping), T, H, D, blk, nb,
        ptr(k_inv.contiguous()), ptr(v_inv.contiguous()), ptr(key_cache), ptr(value_cache),
        stream_handle(key.device),
    )
    _lib.check(rc, "int8_quant_store")


def int8_paged_decode(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    k_aq: torch.Tensor,
    v_aq: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float,
    out: torch.Tensor,
    max_seq_len: int,
) -> torch.Tensor:
    """GQA decode attention over int8 pages; ``query``/``out`` bf16 ``[B, Hq, D]``
    (rows may be strided), ``block_table`` int32 ``[B, >=max_blocks]``,
    ``seq_lens`` int32 ``[B]`` on the device."""
    require_cuda("int8_paged_decode", query, key_cache, value_cache, block_table, seq_lens, out)
    B, Hq, D = query.shape
    nb, blk, H, _ = key_cache.shape
    if B == 0:
        return out
    if query.stride(2) != 1 or query.stride(1) != D or out.stride(2) != 1 or out.stride(1) != D:
        raise RuntimeError("int8_paged_decode: query/out heads must be contiguous [Hq, D] rows")
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    sl = seq_lens if seq_lens.dtype == torch.int32 else seq_lens.to(torch.int32)
    bt = bt.contiguous()
    sl = sl.contiguous()
    lib = _lib.load()
    need = lib.qkv_int8_paged_decode_workspace(B, Hq, H, D, blk, max_seq_len)
    ws = WORKSPACE.get(query.device, need)
    rc = lib.qkv_int8_paged_decode(
        ptr(query), query.stride(0), ptr(key_cache), ptr(value_cache),
        ptr(k_aq.contiguous()), ptr(v_aq.contiguous()), ptr(bt), bt.stride(0), ptr(sl),
        B, Hq, H, D, blk, nb, max_seq_len, float(scale),
        ptr(ws), 0 if ws is None else ws.numel(), ptr(out), out.stride(0),
        stream_handle(query.device),
    )
    _lib.check(rc, "int8_paged_decode")
    return out


__all__ = ["int8_calc_scales", "int8_paged_decode", "int8_quant_store"]
