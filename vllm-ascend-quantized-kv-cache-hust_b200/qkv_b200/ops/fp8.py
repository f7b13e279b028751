"""FP8 per-token-head ops on B200 (libqkv_sm100.so): the store (E4M3 codes +
one fp32 scale per (token, head)), paged decode attention over the pages,
and the dense gather for prompt chunks over cached keys. The store follows
the reference's ``fp8_per_token_head_store`` contract
(ops/triton/per_token_head_store.py:262-294) and the numerics of
``Fp8PerTokenHeadSemantics`` (methods/fp8_per_token_head/semantics.py)."""

from __future__ import annotations

import torch

from . import _lib
from ._torch import WORKSPACE, index_code, ptr, require_cuda, stream_handle

_DTYPES = {torch.float32: _lib.QKV_F32, torch.bfloat16: _lib.QKV_BF16, torch.float16: _lib.QKV_F16}


def _check_views(name: str, data: torch.Tensor, scale: torch.Tensor, kvh: int, d: int) -> None:
    expected = (data.shape[0], data.shape[1], kvh, d)
    if data.dtype != torch.uint8 or tuple(data.shape) != expected or not data.is_contiguous():
        raise RuntimeError(
            f"fp8_per_token_head {name} data cache must be uint8 {expected}, got {tuple(data.shape)} / {data.dtype}."
        )
    es = (data.shape[0], data.shape[1], kvh, 1)
    if scale.dtype != torch.float32 or tuple(scale.shape) != es or not scale.is_contiguous():
        raise RuntimeError(
            f"fp8_per_token_head {name} scale cache must be float32 {es}, got {tuple(scale.shape)} / {scale.dtype}."
        )


def fp8_store(key, value, slot_mapping, k_data, k_scale, v_data, v_scale) -> None:
    """Quantises ``[T, KVH, D]`` K/V per (token, head) and writes codes and
    scales at ``slot_mapping`` (negative slots are skipped)."""
    if key.numel() == 0:
        return
    require_cuda("fp8_store", key, value, slot_mapping, k_data, k_scale, v_data, v_scale)
    T, H, D = key.shape
    if tuple(value.shape) != (T, H, D):
        raise RuntimeError(
            f"fp8_per_token_head key/value token-head grids must match, got key {tuple(key.shape)} vs value "
            f"{tuple(value.shape)}."
        )
    if key.dtype not in _DTYPES or value.dtype != key.dtype:
        raise RuntimeError(f"fp8_store: key/value must share a float dtype, got {key.dtype} / {value.dtype}")
    if tuple(slot_mapping.shape) != (T,):
        raise RuntimeError(
            f"fp8_per_token_head slot_mapping must be 1D of {T} slots, got {tuple(slot_mapping.shape)}."
        )
    _check_views("key", k_data, k_scale, H, D)
    _check_views("value", v_data, v_scale, H, D)
    key, value, slot_mapping = key.contiguous(), value.contiguous(), slot_mapping.contiguous()
    nb, blk = k_data.shape[:2]
    rc = _lib.load().qkv_fp8_store(
        ptr(key), ptr(value), _DTYPES[key.dtype], ptr(slot_mapping), index_code(slot_mapping), T, H, D, blk, nb,
        ptr(k_data), ptr(k_scale), ptr(v_data), ptr(v_scale), stream_handle(key.device),
    )
    _lib.check(rc, "fp8_store")


def fp8_paged_decode(query, k_data, k_scale, v_data, v_scale, block_table, seq_lens, scale, out, max_seq_len):
    """GQA decode attention over the FP8 pages; ``query``/``out`` bf16
    ``[B, Hq, D]`` (rows may be strided), ``block_table`` int32
    ``[B, >= max_blocks]``, ``seq_lens`` int32 ``[B]`` on the device."""
    require_cuda("fp8_paged_decode", query, k_data, block_table, seq_lens, out)
    B, Hq, D = query.shape
    nb, blk, H, _ = k_data.shape
    if B == 0:
        return out
    if query.stride(2) != 1 or query.stride(1) != D or out.stride(2) != 1 or out.stride(1) != D:
        raise RuntimeError("fp8_paged_decode: query/out heads must be contiguous [Hq, D] rows")
    _check_views("key", k_data, k_scale, H, D)
    _check_views("value", v_data, v_scale, H, D)
    bt = (block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)).contiguous()
    sl = (seq_lens if seq_lens.dtype == torch.int32 else seq_lens.to(torch.int32)).contiguous()
    lib = _lib.load()
    need = lib.qkv_fp8_paged_decode_workspace(B, Hq, H, D, blk, max_seq_len)
    ws = WORKSPACE.get(query.device, need)
    rc = lib.qkv_fp8_paged_decode(
        ptr(query), query.stride(0), ptr(k_data), ptr(k_scale), ptr(v_data), ptr(v_scale), ptr(bt), bt.stride(0),
        ptr(sl), B, Hq, H, D, blk, nb, max_seq_len, float(scale), ptr(ws), 0 if ws is None else ws.numel(),
        ptr(out), out.stride(0), stream_handle(query.device),
    )
    _lib.check(rc, "fp8_paged_decode")
    return out


def fp8_dequant_gather(k_data, k_scale, v_data, v_scale, block_table, seq_lens, out_key=None, out_value=None):
    """Dense bf16 ``[sum(seq_lens), KVH, D]`` K/V of whole requests from the
    FP8 pages: row ``sum(seq_lens[:b]) + t`` is position ``t`` of request
    ``b``, ``bf16(code * scale)``; ``seq_lens`` on the host."""
    require_cuda("fp8_dequant_gather", k_data, v_data, block_table)
    nb, blk, H, D = k_data.shape
    B = len(seq_lens)
    total = sum(int(n) for n in seq_lens)
    dev = k_data.device
    out_key = torch.empty(total, H, D, dtype=torch.bfloat16, device=dev) if out_key is None else out_key
    out_value = torch.empty(total, H, D, dtype=torch.bfloat16, device=dev) if out_value is None else out_value
    if B == 0 or total == 0:
        return out_key, out_value
    _check_views("key", k_data, k_scale, H, D)
    _check_views("value", v_data, v_scale, H, D)
    cu = [0]
    for n in seq_lens:
        cu.append(cu[-1] + int(n))
    cu_t = torch.tensor(cu, dtype=torch.int32).to(dev, non_blocking=True)
    sl = torch.tensor([int(n) for n in seq_lens], dtype=torch.int32).to(dev, non_blocking=True)
    bt = (block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)).contiguous()
    rc = _lib.load().qkv_fp8_dequant_gather(
        ptr(k_data), ptr(k_scale), ptr(v_data), ptr(v_scale), ptr(bt), bt.stride(0), ptr(sl), ptr(cu_t), B, H, D,
        blk, nb, total, ptr(out_key), ptr(out_value), stream_handle(dev),
    )
    _lib.check(rc, "fp8_dequant_gather")
    return out_key, out_value


__all__ = ["fp8_dequant_gather", "fp8_paged_decode", "fp8_store"]
