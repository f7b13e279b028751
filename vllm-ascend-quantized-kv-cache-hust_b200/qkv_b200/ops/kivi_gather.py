"""Dense bf16 K/V of whole requests from the KIVI int4 pages and the bf16
residual windows (libqkv_sm100.so): the reference's
``kivi_dequant_gather_cache`` (ops/kivi_gather.py:36-156) followed by its
residual overwrite (methods/kivi_int4/attention_backend.py:849-935)."""

from __future__ import annotations

import torch

from . import _lib
from ._torch import ptr, require_cuda, stream_handle


def kivi_dequant_gather(
    caches: tuple[torch.Tensor, ...],
    residual_key: torch.Tensor | None,
    residual_value: torch.Tensor | None,
    block_table: torch.Tensor,
    seq_lens: list[int],
    res_state: torch.Tensor | None,
    group_size: int,
    out_key: torch.Tensor | None = None,
    out_value: torch.Tensor | None = None,
    cu_seqlens: torch.Tensor | None = None,
    seq_lens_device: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns bf16 ``[sum(seq_lens), KVH, D]`` keys and values: row
    ``sum(seq_lens[:b]) + t`` is position ``t`` of request ``b``.
    ``res_state`` int32 ``[B, 6]`` as for ``kivi_paged_decode`` (None: no
    windows); ``seq_lens`` on the host. ``cu_seqlens`` (int32 ``[B + 1]``
    prefix sums) and ``seq_lens_device`` (int32 ``[B]``) already on the device
    skip the per-call upload, so the call can be captured in a CUDA graph."""
    kq, ks, km, vq, vs, vm = caches
    require_cuda("kivi_dequant_gather", kq, vq, block_table)
    nb, H, D, wpb = kq.shape
    blk = wpb * 8
    B = len(seq_lens)
    total = sum(int(n) for n in seq_lens)
    dev = kq.device
    if out_key is None:
        out_key = torch.empty(total, H, D, dtype=torch.bfloat16, device=dev)
    if out_value is None:
        out_value = torch.empty(total, H, D, dtype=torch.bfloat16, device=dev)
    if B == 0 or total == 0:
        return out_key, out_value
    if cu_seqlens is None:
        cu = [0]
        for n in seq_lens:
            cu.append(cu[-1] + int(n))
        cu_t = torch.tensor(cu, dtype=torch.int32).to(dev, non_blocking=True)
    else:
        cu_t = cu_seqlens
    if seq_lens_device is None:
        sl = torch.tensor([int(n) for n in seq_lens], dtype=torch.int32).to(dev, non_blocking=True)
    else:
        sl = seq_lens_device
    for name, t, n in (("cu_seqlens", cu_t, B + 1), ("seq_lens_device", sl, B)):
        if t.dtype != torch.int32 or t.numel() != n or t.device != dev:
            raise RuntimeError(f"kivi_dequant_gather: {name} must be int32 [{n}] on the cache's device")
    for name, t in (("out_key", out_key), ("out_value", out_value)):
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.shape[0] < total or tuple(t.shape[1:]) != (H, D):
            raise RuntimeError(f"kivi_dequant_gather: {name} must be contiguous bf16 [>= {total}, {H}, {D}]")
    bt = (block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)).contiguous()
    rows = cap = 0
    if res_state is not None:
        if residual_key is None or residual_value is None:
            raise RuntimeError("kivi_dequant_gather: res_state needs the residual buffers")
        rows, cap = residual_key.shape[:2]
        res_state = res_state.contiguous()
    rc = _lib.load().qkv_kivi_dequant_gather(
        ptr(kq), ptr(ks), ptr(km), ptr(vq), ptr(vs), ptr(vm),
        ptr(residual_key), ptr(residual_value), rows, cap,
        ptr(bt), bt.stride(0), ptr(sl), ptr(cu_t), ptr(res_state), B,
        H, D, group_size, blk, nb, total, ptr(out_key), ptr(out_value),
        stream_handle(dev),
    )
    _lib.check(rc, "kivi_dequant_gather")
    return out_key, out_value


__all__ = ["kivi_dequant_gather"]
