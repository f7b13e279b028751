"""One KIVI decode step in one native call (``qkv_kivi_decode_step``): the
DecodeOnly branch of the reference's forward
(methods/kivi_int4/attention_backend.py:1006-1040 — window writes, window
sync, paged decode attention) with the planning in C++, every index staged
through one pinned buffer and one host-to-device copy, and no host sync."""

from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._torch import WORKSPACE, ptr, require_cuda, stream_handle


class KiviDecodeStep:
    """Owns the native step runtime (pinned and device staging buffers) of one
    attention layer. ``bind`` checks and records the per-layer arguments (the
    window planner, the six cache views, the residual rings) once; ``run``
    takes only what changes from step to step."""

    def __init__(self) -> None:
        self._lib = _lib.load()
        self._handle = self._lib.qkv_kivi_step_create()
        if not self._handle:
            raise RuntimeError("qkv_kivi_step_create failed")
        self._static = None
        self._ws_key = None
        self._ws_need = 0

    def __del__(self) -> None:
        h, self._handle = getattr(self, "_handle", None), None
        if h:
            self._lib.qkv_kivi_step_destroy(h)

    def bind(self, window_handle: int, caches: tuple[torch.Tensor, ...], residual_key: torch.Tensor,
             residual_value: torch.Tensor, group_size: int, scale: float) -> None:
        """``caches`` the six KIVI views; rings bf16 ``[rows, capacity, KVH, D]``."""
        kq, ks, km, vq, vs, vm = caches
        require_cuda("kivi_decode_step", kq, ks, km, vq, vs, vm, residual_key, residual_value)
        if residual_key.dtype != torch.bfloat16 or residual_value.dtype != torch.bfloat16:
            raise RuntimeError("kivi_decode_step: residual windows must be bf16")
        nb, H, D, wpb = kq.shape
        self._window = window_handle
        self._geom = (H, D, wpb * 8, nb, group_size, float(scale))
        self._static = (ptr(kq), ptr(ks), ptr(km), ptr(vq), ptr(vs), ptr(vm), ptr(residual_key),
                        ptr(residual_value))
        self._device = kq.device

    def run(
        self,
        rows: np.ndarray,
        slots: np.ndarray,
        seq_lens: np.ndarray,
        block_table_host: np.ndarray,
        block_table: torch.Tensor | None,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        out: torch.Tensor,
    ) -> torch.Tensor:
        """``rows`` / ``slots`` int64 and ``seq_lens`` int32 host arrays of
        the batch; ``block_table_host`` int32 ``[B, cols]`` host,
        ``block_table`` the same table int32 on the device, or None to let
        the step stage the host table with its indices (one copy for the
        whole step); ``query`` / ``out`` bf16
        ``[B, Hq, D]``; ``key`` / ``value`` the new tokens, bf16
        ``[B, KVH, D]`` contiguous on the device."""
        if self._static is None:
            raise RuntimeError("kivi_decode_step: bind() the layer's caches first")
        H, D, blk, nb, group_size, scale = self._geom
        require_cuda("kivi_decode_step", query, key, value, out)
        B, Hq = query.shape[0], query.shape[1]
        for name, t in (("query", query), ("out", out)):
            if t.dtype != torch.bfloat16 or t.stride(2) != 1 or t.stride(1) != D:
                raise RuntimeError(f"kivi_decode_step: {name} must be bf16 with contiguous [Hq, D] rows")
        for name, t in (("key", key), ("value", value)):
            if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.shape != (B, H, D):
                raise RuntimeError(f"kivi_decode_step: {name} must be contiguous bf16 [{B}, {H}, {D}]")
        if block_table is not None:
            require_cuda("kivi_decode_step", block_table)
            if block_table.dtype != torch.int32 or block_table.stride(1) != 1:
                raise RuntimeError("kivi_decode_step: block_table must be int32 with contiguous rows")
        if block_table_host.dtype != np.int32 or not block_table_host.flags.c_contiguous:
            block_table_host = np.ascontiguousarray(block_table_host, dtype=np.int32)
        max_len = max(int(seq_lens.max()) if seq_lens.size else 1, 1)
        # the decode plan (hence the workspace) only changes with the page count
        ws_key = (B, Hq, (max_len + blk - 1) // blk)
        if ws_key != self._ws_key:
            self._ws_need = self._lib.qkv_kivi_paged_decode_workspace(B, Hq, H, D, group_size, blk, max_len)
            self._ws_key = ws_key
        ws = WORKSPACE.get(self._device, self._ws_need)
        rc = self._lib.qkv_kivi_decode_step(
            self._handle, self._window, B, rows.ctypes.data, slots.ctypes.data, seq_lens.ctypes.data,
            block_table_host.ctypes.data, block_table_host.shape[1],
            0 if block_table is None else block_table.data_ptr(), 0 if block_table is None else block_table.stride(0),
            query.data_ptr(), query.stride(0), key.data_ptr(), value.data_ptr(), *self._static, Hq, H, D,
            group_size, blk, nb, scale, ptr(ws), 0 if ws is None else ws.numel(), out.data_ptr(), out.stride(0),
            stream_handle(self._device),
        )
        _lib.check(rc, "kivi_decode_step")
        return out


__all__ = ["KiviDecodeStep"]
