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
    attention layer."""

    def __init__(self) -> None:
        self._lib = _lib.load()
        self._handle = self._lib.qkv_kivi_step_create()
        if not self._handle:
            raise RuntimeError("qkv_kivi_step_create failed")

    def __del__(self) -> None:
        h, self._handle = getattr(self, "_handle", None), None
        if h:
            self._lib.qkv_kivi_step_destroy(h)

    def run(
        self,
        window_handle: int,
        rows: np.ndarray,
        slots: np.ndarray,
        seq_lens: np.ndarray,
        block_table_host: np.ndarray,
        block_table: torch.Tensor,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        caches: tuple[torch.Tensor, ...],
        residual_key: torch.Tensor,
        residual_value: torch.Tensor,
        group_size: int,
        scale: float,
        out: torch.Tensor,
    ) -> torch.Tensor:
        """``rows`` / ``slots`` int64 and ``seq_lens`` int32 host arrays of
        the batch; ``block_table_host`` int64 ``[B, cols]`` host,
        ``block_table`` int32 on the device; ``query`` / ``out`` bf16
        ``[B, Hq, D]``; ``key`` / ``value`` the new tokens, bf16
        ``[B, KVH, D]`` contiguous on the device."""
        kq, ks, km, vq, vs, vm = caches
        require_cuda("kivi_decode_step", query, key, value, kq, residual_key, block_table, out)
        B, Hq, D = query.shape
        nb, H, _, wpb = kq.shape
        blk = wpb * 8
        for name, t in (("query", query), ("out", out)):
            if t.dtype != torch.bfloat16 or t.stride(2) != 1 or t.stride(1) != D:
                raise RuntimeError(f"kivi_decode_step: {name} must be bf16 with contiguous [Hq, D] rows")
        for name, t in (("key", key), ("value", value)):
            if t.dtype != torch.bfloat16 or not t.is_contiguous() or tuple(t.shape) != (B, H, D):
                raise RuntimeError(f"kivi_decode_step: {name} must be contiguous bf16 [{B}, {H}, {D}]")
        if residual_key.dtype != torch.bfloat16 or residual_value.dtype != torch.bfloat16:
            raise RuntimeError("kivi_decode_step: residual windows must be bf16")
        if block_table.dtype != torch.int32 or block_table.stride(1) != 1:
            raise RuntimeError("kivi_decode_step: block_table must be int32 with contiguous rows")
        bth = np.ascontiguousarray(block_table_host, dtype=np.int64)
        max_len = int(seq_lens.max()) if seq_lens.size else 1
        need = self._lib.qkv_kivi_paged_decode_workspace(B, Hq, H, D, group_size, blk, max(max_len, 1))
        ws = WORKSPACE.get(query.device, need)
        rc = self._lib.qkv_kivi_decode_step(
            self._handle, window_handle, B, rows.ctypes.data, slots.ctypes.data, seq_lens.ctypes.data,
            bth.ctypes.data, bth.shape[1], ptr(block_table), block_table.stride(0), ptr(query), query.stride(0),
            ptr(key), ptr(value), ptr(kq), ptr(ks), ptr(km), ptr(vq), ptr(vs), ptr(vm), ptr(residual_key),
            ptr(residual_value), Hq, H, D, group_size, blk, nb, float(scale), ptr(ws),
            0 if ws is None else ws.numel(), ptr(out), out.stride(0), stream_handle(query.device),
        )
        _lib.check(rc, "kivi_decode_step")
        return out


__all__ = ["KiviDecodeStep"]
