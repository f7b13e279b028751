"""Host-side layout validators run before every KIVI kernel launch.

Same rules and error messages as the reference's shared validators
(ops/kivi_layout.py:11-238 of vllm_ascend_quantized_kv_cache), so callers that
match on those messages keep working. The checks run on tensor metadata; the
two that inspect values (slot groups, block-table coverage) do one small
device->host read, exactly where the reference does.
"""

from __future__ import annotations

import torch


def _check_same_device(name: str, tensor: torch.Tensor, ref: torch.Tensor) -> None:
    if tensor.device != ref.device:
        raise RuntimeError(f"{name} must be on device {ref.device}, got {tensor.device}.")


def _check_contiguous(name: str, tensor: torch.Tensor) -> None:
    if not tensor.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous.")


def _check_value_cache_layout(v_quant_cache, v_scale_cache, v_mn_cache, *, num_kv_heads, head_size, group_size):
    """reference ops/kivi_layout.py:25-65"""
    if v_quant_cache.ndim != 4:
        raise RuntimeError(f"v_quant_cache must be 4D, got shape={tuple(v_quant_cache.shape)}.")
    if v_scale_cache.ndim != 4 or v_mn_cache.ndim != 4:
        raise RuntimeError(
            "v_scale_cache and v_mn_cache must be 4D, got "
            f"{tuple(v_scale_cache.shape)} and {tuple(v_mn_cache.shape)}."
        )
    nb, block, heads, packed = v_quant_cache.shape
    want_q = (nb, block, num_kv_heads, head_size // 8)
    want_s = (nb, block, num_kv_heads, head_size // group_size)
    if tuple(v_quant_cache.shape) != want_q:
        raise RuntimeError(f"v_quant_cache layout mismatch: got {tuple(v_quant_cache.shape)}, expected {want_q}.")
    if tuple(v_scale_cache.shape) != want_s:
        raise RuntimeError(f"v_scale_cache layout mismatch: got {tuple(v_scale_cache.shape)}, expected {want_s}.")
    if tuple(v_mn_cache.shape) != want_s:
        raise RuntimeError(f"v_mn_cache layout mismatch: got {tuple(v_mn_cache.shape)}, expected {want_s}.")
    if packed != head_size // 8 or heads != num_kv_heads:
        raise RuntimeError("v_quant_cache head layout does not match input value tensor.")


def _check_key_cache_layout(k_quant_cache, k_scale_cache, k_mn_cache, *, num_kv_heads, head_size, group_size) -> int:
    """reference ops/kivi_layout.py:68-108; returns the block size."""
    if k_quant_cache.ndim != 4:
        raise RuntimeError(f"k_quant_cache must be 4D, got shape={tuple(k_quant_cache.shape)}.")
    if k_scale_cache.ndim != 4 or k_mn_cache.ndim != 4:
        raise RuntimeError(
            "k_scale_cache and k_mn_cache must be 4D, got "
            f"{tuple(k_scale_cache.shape)} and {tuple(k_mn_cache.shape)}."
        )
    nb, heads, hs, packed_block = k_quant_cache.shape
    block = packed_block * 8
    want_q = (nb, num_kv_heads, head_size, block // 8)
    want_s = (nb, num_kv_heads, head_size, block // group_size)
    if tuple(k_quant_cache.shape) != want_q:
        raise RuntimeError(f"k_quant_cache layout mismatch: got {tuple(k_quant_cache.shape)}, expected {want_q}.")
    if tuple(k_scale_cache.shape) != want_s:
        raise RuntimeError(f"k_scale_cache layout mismatch: got {tuple(k_scale_cache.shape)}, expected {want_s}.")
    if tuple(k_mn_cache.shape) != want_s:
        raise RuntimeError(f"k_mn_cache layout mismatch: got {tuple(k_mn_cache.shape)}, expected {want_s}.")
    if heads != num_kv_heads or hs != head_size:
        raise RuntimeError("k_quant_cache head layout does not match input key tensor.")
    return block


def _check_slot_mapping(slot_mapping: torch.Tensor, num_tokens: int) -> None:
    """reference ops/kivi_layout.py:111-124"""
    if slot_mapping.ndim != 1:
        raise RuntimeError(f"slot_mapping must be 1D, got shape={tuple(slot_mapping.shape)}.")
    if slot_mapping.numel() != num_tokens:
        raise RuntimeError(
            f"slot_mapping length must match num_tokens, got {slot_mapping.numel()} vs {num_tokens}."
        )
    if slot_mapping.dtype not in (torch.int32, torch.int64):
        raise RuntimeError(f"slot_mapping must be int32/int64, got {slot_mapping.dtype}.")


def _check_key_slot_groups(slot_mapping: torch.Tensor, *, block_size: int, group_size: int) -> None:
    """Whole-group key flush gate (reference ops/kivi_layout.py:127-163):
    every group of ``group_size`` slots is contiguous, group aligned and
    inside one cache block. The same rule as ``is_aligned_key_window``."""
    if bool((slot_mapping < 0).any()):
        raise RuntimeError("kivi_pack_key_cache requires all slot_mapping entries to be valid.")
    groups = slot_mapping.view(-1, group_size)
    first = groups[:, :1]
    offsets = torch.arange(group_size, device=slot_mapping.device, dtype=slot_mapping.dtype).view(1, -1)
    if not bool((groups == first + offsets).all()):
        raise RuntimeError("kivi_pack_key_cache requires each token group to map to contiguous slots.")
    if not bool(((first % group_size) == 0).all()):
        raise RuntimeError("kivi_pack_key_cache requires each token group to be group-size aligned.")
    if not bool(((groups // block_size) == (first // block_size)).all()):
        raise RuntimeError("kivi_pack_key_cache requires each token group to stay within one cache block.")


def _check_block_table(block_table: torch.Tensor) -> None:
    if block_table.ndim != 2:
        raise RuntimeError(f"block_table must be 2D, got shape={tuple(block_table.shape)}.")
    if block_table.dtype not in (torch.int32, torch.int64):
        raise RuntimeError(f"block_table must be int32/int64, got {block_table.dtype}.")


def _check_seq_lens(seq_lens: torch.Tensor, batch_size: int) -> None:
    if seq_lens.ndim != 1:
        raise RuntimeError(f"seq_lens must be 1D, got shape={tuple(seq_lens.shape)}.")
    if seq_lens.numel() != batch_size:
        raise RuntimeError(f"seq_lens length must match batch size, got {seq_lens.numel()} vs {batch_size}.")
    if seq_lens.dtype not in (torch.int32, torch.int64):
        raise RuntimeError(f"seq_lens must be int32/int64, got {seq_lens.dtype}.")


def _check_paged_metadata(block_table, seq_lens: list[int], *, num_blocks: int, block_size: int) -> None:
    """Coverage and range of the live block-table entries (the rules of the
    reference's ``_check_dequant_gather_metadata``, ops/kivi_layout.py:187-238),
    evaluated on a host copy of the table."""
    _check_block_table(block_table)
    batch = len(seq_lens)
    if block_table.shape[0] < batch:
        raise RuntimeError(f"block_table batch size must match seq_lens, got {block_table.shape[0]} vs {batch}.")
    if batch == 0:
        return
    max_len = max(int(s) for s in seq_lens)
    if max_len > block_table.shape[1] * block_size:
        raise RuntimeError(
            "block_table does not cover the longest KIVI sequence: "
            f"max_seq_len={max_len}, max_blocks={block_table.shape[1]}, block_size={block_size}."
        )
    bt = block_table[:batch].cpu() if block_table.is_cuda else block_table[:batch]
    counts = torch.tensor([(int(s) + block_size - 1) // block_size for s in seq_lens])
    live = torch.arange(bt.shape[1]).unsqueeze(0) < counts.unsqueeze(1)
    ids = bt[live]
    if bool((ids < 0).any()):
        raise RuntimeError("KIVI block_table has invalid block ids for live tokens.")
    if bool((ids >= num_blocks).any()):
        raise RuntimeError("KIVI block_table references blocks outside the int4 cache.")


__all__ = [
    "_check_block_table",
    "_check_contiguous",
    "_check_key_cache_layout",
    "_check_key_slot_groups",
    "_check_paged_metadata",
    "_check_same_device",
    "_check_seq_lens",
    "_check_slot_mapping",
    "_check_value_cache_layout",
]
