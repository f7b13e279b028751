"""Device side of a residual-window plan (libqkv_sm100.so): gather the token
rows a plan names — ring lanes or new tokens — and scatter rows into ring
lanes, both sides in one launch each. Replaces the per-step index_select /
index_copy_ of the reference's window writes
(methods/kivi_int4/attention_backend.py:411-462)."""

from __future__ import annotations

import torch

from . import _lib
from ._torch import ptr, require_cuda, stream_handle


def _row_bytes(ring: torch.Tensor) -> int:
    return ring[0, 0].numel() * ring.element_size()


def _check_ring(name: str, ring: torch.Tensor) -> None:
    if not ring.is_contiguous():
        raise RuntimeError(f"{name}: residual rings must be contiguous")
    if _row_bytes(ring) % 16:
        raise RuntimeError(f"{name}: a ring row must be a multiple of 16 bytes")


def kivi_window_gather(
    ring_key: torch.Tensor,
    ring_value: torch.Tensor,
    new_key: torch.Tensor | None,
    new_value: torch.Tensor | None,
    key_src: torch.Tensor,
    value_src: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Rings ``[rows, capacity, KVH, D]``; new tokens ``[T, KVH, D]`` of the
    rings' dtype (None when no source names one); sources int64 on the device
    (s >= 0: flat lane ``row * capacity + lane``, s < 0: new token ``-1 - s``).
    Returns ``[len(key_src), KVH, D]`` and ``[len(value_src), KVH, D]``."""
    require_cuda("kivi_window_gather", ring_key, ring_value, key_src, value_src)
    _check_ring("kivi_window_gather", ring_key)
    _check_ring("kivi_window_gather", ring_value)
    shape = tuple(ring_key.shape[2:])
    out_k = torch.empty((key_src.numel(), *shape), dtype=ring_key.dtype, device=ring_key.device)
    out_v = torch.empty((value_src.numel(), *shape), dtype=ring_value.dtype, device=ring_value.device)
    if key_src.numel() + value_src.numel() == 0:
        return out_k, out_v
    for name, t, ring in (("new_key", new_key, ring_key), ("new_value", new_value, ring_value)):
        if t is not None and (t.dtype != ring.dtype or not t.is_contiguous() or tuple(t.shape[1:]) != shape):
            raise RuntimeError(f"kivi_window_gather: {name} must be contiguous {ring.dtype} [T, {shape}]")
    n_new = 0
    if new_key is not None and new_value is not None:
        n_new = min(new_key.shape[0], new_value.shape[0])
    elif new_key is not None or new_value is not None:
        # one side carries no new tokens: its sources may only name ring lanes
        n_new = (new_key if new_key is not None else new_value).shape[0]
    nk_src = new_key if new_key is not None else new_value
    nv_src = new_value if new_value is not None else new_key
    lanes = ring_key.shape[0] * ring_key.shape[1]
    rc = _lib.load().qkv_kivi_window_gather(
        ptr(ring_key), ptr(ring_value), lanes, ptr(nk_src), ptr(nv_src), n_new,
        ptr(key_src), key_src.numel(), ptr(value_src), value_src.numel(), _row_bytes(ring_key),
        ptr(out_k), ptr(out_v), stream_handle(ring_key.device),
    )
    _lib.check(rc, "kivi_window_gather")
    return out_k, out_v


def kivi_window_scatter(
    ring_key: torch.Tensor,
    ring_value: torch.Tensor,
    key_lanes: torch.Tensor,
    key_rows: torch.Tensor,
    value_lanes: torch.Tensor,
    value_rows: torch.Tensor,
) -> None:
    """``ring_key.view(-1, KVH, D)[key_lanes[i]] = key_rows[i]``, likewise for
    values, in one launch."""
    require_cuda("kivi_window_scatter", ring_key, ring_value, key_lanes, value_lanes)
    _check_ring("kivi_window_scatter", ring_key)
    _check_ring("kivi_window_scatter", ring_value)
    if key_lanes.numel() + value_lanes.numel() == 0:
        return
    for name, rows, lanes, ring in (("key", key_rows, key_lanes, ring_key), ("value", value_rows, value_lanes,
                                                                             ring_value)):
        if rows.shape[0] != lanes.numel() or rows.dtype != ring.dtype or not rows.is_contiguous():
            raise RuntimeError(f"kivi_window_scatter: {name} rows must be contiguous {ring.dtype} [len(lanes), ...]")
    n = ring_key.shape[0] * ring_key.shape[1]
    rc = _lib.load().qkv_kivi_window_scatter(
        ptr(ring_key), ptr(ring_value), n, ptr(key_lanes), key_lanes.numel(), ptr(key_rows),
        ptr(value_lanes), value_lanes.numel(), ptr(value_rows), _row_bytes(ring_key),
        stream_handle(ring_key.device),
    )
    _lib.check(rc, "kivi_window_scatter")


__all__ = ["kivi_window_gather", "kivi_window_scatter"]
