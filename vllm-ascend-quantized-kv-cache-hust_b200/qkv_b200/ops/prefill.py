"""Prompt attention over full-precision K/V (TND layout) on B200.

Replaces the FIA calls of the all-new prefill branches of both methods
(methods/kivi_int4/attention_backend.py:1232-1266, :1315-1338;
methods/int8_dynamic/attention_backend.py:246-368): causal attention aligned
to the end of each request's keys (FIA sparse_mode 3)."""

from __future__ import annotations

import torch

from . import _lib
from ._torch import WORKSPACE, ptr, require_cuda, stream_handle


def _cumulative(lengths, device) -> torch.Tensor:
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + int(n))
    return torch.tensor(cu, dtype=torch.int32).to(device, non_blocking=True)


def dense_prefill(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    q_lens: list[int],
    kv_lens: list[int],
    scale: float,
    out: torch.Tensor,
    causal: bool = True,
    cu_seqlens_q: torch.Tensor | None = None,
    cu_seqlens_k: torch.Tensor | None = None,
) -> torch.Tensor:
    """``query``/``out`` bf16 ``[sum q_lens, Hq, D]`` (contiguous), ``key``/
    ``value`` bf16 ``[sum kv_lens, KVH, D]``; per-request lengths on host.
    ``cu_seqlens_q`` / ``cu_seqlens_k`` (int32 ``[B + 1]`` on the device, the
    prefix sums of the lengths) skip the per-call upload, so the call can be
    captured in a CUDA graph."""
    require_cuda("dense_prefill", query, key, value, out)
    total_q, Hq, D = query.shape
    H = key.shape[1]
    if total_q == 0 or not q_lens:
        return out
    for name, t in (("query", query), ("key", key), ("value", value), ("out", out)):
        if t.dtype != torch.bfloat16:
            raise RuntimeError(f"dense_prefill: {name} must be bfloat16, got {t.dtype}")
        if not t.is_contiguous():
            raise RuntimeError(f"dense_prefill: {name} must be contiguous")
    if sum(int(n) for n in q_lens) != total_q:
        raise RuntimeError("dense_prefill: q_lens do not sum to the query rows")
    cu_q = _cumulative(q_lens, query.device) if cu_seqlens_q is None else cu_seqlens_q
    cu_k = _cumulative(kv_lens, query.device) if cu_seqlens_k is None else cu_seqlens_k
    for name, t in (("cu_seqlens_q", cu_q), ("cu_seqlens_k", cu_k)):
        if t.dtype != torch.int32 or t.numel() != len(q_lens) + 1 or t.device != query.device:
            raise RuntimeError(f"dense_prefill: {name} must be int32 [B + 1] on the query's device")
    max_kv = max(int(n) for n in kv_lens)
    lib = _lib.load()
    need = lib.qkv_dense_prefill_workspace(total_q, Hq, H, D, max_kv)
    ws = WORKSPACE.get(query.device, need)
    total_k = sum(int(n) for n in kv_lens)
    if key.shape[0] < total_k or value.shape[0] < total_k:
        raise RuntimeError("dense_prefill: kv_lens exceed the key / value rows")
    rc = lib.qkv_dense_prefill(
        ptr(query), ptr(key), ptr(value), ptr(cu_q), ptr(cu_k), len(q_lens), total_q, total_k, Hq, H, D,
        int(bool(causal)), max_kv, float(scale), ptr(ws), 0 if ws is None else ws.numel(), ptr(out),
        stream_handle(query.device),
    )
    _lib.check(rc, "dense_prefill")
    return out


__all__ = ["dense_prefill"]
