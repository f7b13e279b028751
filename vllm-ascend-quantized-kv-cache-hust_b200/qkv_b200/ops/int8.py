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


def int8_dequant_gather(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    k_aq: torch.Tensor,
    v_aq: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: list[int],
    out_key: torch.Tensor | None = None,
    out_value: torch.Tensor | None = None,
    cu_seqlens: torch.Tensor | None = None,
    seq_lens_device: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Dense bf16 ``[sum(seq_lens), KVH, D]`` K/V from the int8 pages
    (``_dequant_int8_paged_kv_to_dense``, attention_backend.py:370-404): row
    ``sum(seq_lens[:b]) + t`` is position ``t`` of request ``b``, dequantised
    as ``code * aq`` in bf16. ``seq_lens`` on the host; ``cu_seqlens`` /
    ``seq_lens_device`` (int32, already on the device) make the call
    capturable in a CUDA graph."""
    require_cuda("int8_dequant_gather", key_cache, value_cache, block_table)
    nb, blk, H, D = key_cache.shape
    B = len(seq_lens)
    total = sum(int(n) for n in seq_lens)
    dev = key_cache.device
    if out_key is None:
        out_key = torch.empty(total, H, D, dtype=torch.bfloat16, device=dev)
    if out_value is None:
        out_value = torch.empty(total, H, D, dtype=torch.bfloat16, device=dev)
    if B == 0 or total == 0:
        return out_key, out_value
    cu_t = cu_seqlens
    if cu_t is None:
        cu = [0]
        for n in seq_lens:
            cu.append(cu[-1] + int(n))
        cu_t = torch.tensor(cu, dtype=torch.int32).to(dev, non_blocking=True)
    sl = seq_lens_device
    if sl is None:
        sl = torch.tensor([int(n) for n in seq_lens], dtype=torch.int32).to(dev, non_blocking=True)
    for name, t, n in (("cu_seqlens", cu_t, B + 1), ("seq_lens_device", sl, B)):
        if t.dtype != torch.int32 or t.numel() != n or t.device != dev:
            raise RuntimeError(f"int8_dequant_gather: {name} must be int32 [{n}] on the cache's device")
    for name, t in (("out_key", out_key), ("out_value", out_value)):
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.shape[0] < total or tuple(t.shape[1:]) != (H, D):
            raise RuntimeError(f"int8_dequant_gather: {name} must be contiguous bf16 [>= {total}, {H}, {D}]")
    bt = (block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)).contiguous()
    rc = _lib.load().qkv_int8_dequant_gather(
        ptr(key_cache), ptr(value_cache), ptr(k_aq.contiguous()), ptr(v_aq.contiguous()), ptr(bt), bt.stride(0),
        ptr(sl), ptr(cu_t), B, H, D, blk, nb, total, ptr(out_key), ptr(out_value), stream_handle(dev),
    )
    _lib.check(rc, "int8_dequant_gather")
    return out_key, out_value


__all__ = ["int8_calc_scales", "int8_dequant_gather", "int8_paged_decode", "int8_quant_store"]
