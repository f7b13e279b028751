"""Fused KIVI INT4 paged decode attention on B200 (libqkv_sm100.so).

Replaces the reference's read path — ``kivi_dequant_gather_cache``
(ops/kivi_gather.py:36-156) + residual tail overwrite + FIA TND
(methods/kivi_int4/attention_backend.py:849-935, :1193-1230) — with one kernel
that streams the int4 pages, dequantises in registers and merges the bf16
residual window into the same online softmax."""

from __future__ import annotations

import ctypes
from typing import NamedTuple

import torch

from . import _lib
from ._torch import WORKSPACE, ptr, require_cuda, stream_handle

RES_STATE_FIELDS = 6  # row, k_start, k_len, v_start, v_len, end


def kivi_paged_decode(
    query: torch.Tensor,
    caches: tuple[torch.Tensor, ...],
    residual_key: torch.Tensor | None,
    residual_value: torch.Tensor | None,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    res_state: torch.Tensor | None,
    group_size: int,
    scale: float,
    out: torch.Tensor,
    max_seq_len: int,
    partials: bool = False,
):
    """Decode attention for ``query`` bf16 ``[B, Hq, D]`` into ``out``.

    ``caches`` are the six views ``(k_quant, k_scale, k_mn, v_quant, v_scale,
    v_mn)``; ``residual_key/value`` bf16 ``[rows, cap, KVH, D]``;
    ``res_state`` int32 ``[B, 6]`` (row, k_start, k_len, v_start, v_len, end);
    ``block_table`` int32 ``[B, >=max_blocks]``; ``seq_lens`` int32 ``[B]``.
    With ``partials=True`` the split partials stay in the workspace for a
    combining consumer and a ``DecodePartials`` is returned
    (``qkv_kivi_paged_decode_partials``)."""
    kq, ks, km, vq, vs, vm = caches
    require_cuda("kivi_paged_decode", query, kq, vq, block_table, seq_lens, out)
    B, Hq, D = query.shape
    nb, H, _, wpb = kq.shape
    blk = wpb * 8
    if B == 0:
        return out
    if query.stride(2) != 1 or query.stride(1) != D or out.stride(2) != 1 or out.stride(1) != D:
        raise RuntimeError("kivi_paged_decode: query/out heads must be contiguous [Hq, D] rows")
    if query.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise RuntimeError("kivi_paged_decode: query/out must be bfloat16")
    bt = (block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)).contiguous()
    sl = (seq_lens if seq_lens.dtype == torch.int32 else seq_lens.to(torch.int32)).contiguous()
    rows = cap = 0
    if res_state is not None:
        if residual_key is None or residual_value is None:
            raise RuntimeError("kivi_paged_decode: res_state needs the residual buffers")
        if residual_key.dtype != torch.bfloat16 or residual_value.dtype != torch.bfloat16:
            raise RuntimeError("kivi_paged_decode: residual buffers must be bfloat16")
        rows, cap = residual_key.shape[:2]
        res_state = res_state.contiguous()
        if res_state.dtype != torch.int32 or tuple(res_state.shape) != (B, RES_STATE_FIELDS):
            raise RuntimeError(f"kivi_paged_decode: res_state must be int32 [{B}, {RES_STATE_FIELDS}]")
    lib = _lib.load()
    need = lib.qkv_kivi_paged_decode_workspace(B, Hq, H, D, group_size, blk, max_seq_len)
    ws = WORKSPACE.get(query.device, need)
    args = (
        ptr(query), query.stride(0), ptr(kq), ptr(ks), ptr(km), ptr(vq), ptr(vs), ptr(vm),
        ptr(residual_key), ptr(residual_value), rows, cap,
        ptr(bt), bt.stride(0), ptr(sl), ptr(res_state),
        B, Hq, H, D, group_size, blk, nb, max_seq_len, float(scale),
        ptr(ws), 0 if ws is None else ws.numel(), ptr(out), out.stride(0),
    )
    if not partials:
        _lib.check(lib.qkv_kivi_paged_decode(*args, stream_handle(query.device)), "kivi_paged_decode")
        return out
    splits = ctypes.c_int(1)
    rc = lib.qkv_kivi_paged_decode_partials(*args, ctypes.byref(splits), stream_handle(query.device))
    _lib.check(rc, "kivi_paged_decode_partials")
    return DecodePartials(splits.value, ws, B, Hq, D)


class DecodePartials(NamedTuple):
    """Split partials a decode left in ``workspace`` for a combining consumer
    (``PeerGather.gather_partials``): ``[B, Hq, splits, D]`` fp32 sums, then
    ``[B, Hq, splits, 2]`` (max, sum); splits == 1 means ``out`` was written."""

    splits: int
    workspace: torch.Tensor | None
    batch: int
    num_heads: int
    head_size: int

    def acc_ptr(self) -> int:
        return self.workspace.data_ptr()

    def ml_ptr(self) -> int:
        return self.workspace.data_ptr() + self.batch * self.num_heads * self.splits * self.head_size * 4


__all__ = ["RES_STATE_FIELDS", "DecodePartials", "kivi_paged_decode"]
