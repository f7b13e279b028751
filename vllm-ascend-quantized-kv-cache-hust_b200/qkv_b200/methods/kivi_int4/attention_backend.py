"""KIVI INT4 attention implementation for B200 (the plugin-owned mixin).

Same role, method names, state and error behaviour as the reference's
``AscendKiviInt4AttentionBackendMixin`` (methods/kivi_int4/attention_backend.py
of vllm_ascend_quantized_kv_cache): the adapter mixes it over the live host
``AscendAttentionBackendImpl``; it binds the two host byte buffers as the six
KIVI views, keeps one residual-window row per live request, writes K/V through
the window into the int4 history and computes attention.

What runs where:
* residual windows: bf16 ring buffers on the cache device; slot bookkeeping on
  the host (``window.WindowPlanner``), applied once per forward;
* int4 history writes: ``qkv_kivi_pack_key`` / ``qkv_kivi_pack_value``;
* decode attention: ``qkv_kivi_paged_decode`` reads int4 pages and the bf16
  window directly (no dense K/V copy);
* prompt attention over raw K/V: ``qkv_dense_prefill``;
* attention over history for multi-token rows (cache hits, chunked prefill
  with history): ``qkv_kivi_paged_decode`` with one row per query token and
  its causal length.
The reference refuses chunked prefill with history (RuntimeError at
attention_backend.py:1062-1069); this implementation serves it with the
semantics of the reference's generic branch (:1157-1191).
"""

from __future__ import annotations

from typing import Any

import numpy as np
import torch

from .byte_cache import kivi_byte_cache_layout, kivi_caches_from_byte_tensors
from .geometry import validate_kivi_geometry
from .window import SidePlan, WindowPlanner, is_aligned_key_window, ordered_slots


def _attn_state_name(attn_metadata: Any) -> str:
    state = getattr(attn_metadata, "attn_state", None)
    if state is None:
        return "UNKNOWN"
    return getattr(state, "name", None) or str(state)


def _host_i64(x, n: int) -> np.ndarray:
    """First ``n`` entries of an index tensor / list as host int64 (a device
    tensor is read back, as the reference's ``.tolist()`` does)."""
    if isinstance(x, torch.Tensor):
        t = x[:n]
        if t.is_cuda:
            t = t.cpu()
        return t.numpy().astype(np.int64, copy=False).reshape(-1)
    return np.asarray(x, dtype=np.int64).reshape(-1)[:n]


def _host_list(x) -> list[int]:
    if isinstance(x, torch.Tensor):
        return [int(v) for v in x.tolist()]
    return [int(v) for v in x]


class AscendKiviInt4AttentionBackendMixin:
    """KIVI INT4 (int4 history + bf16 residual window) attention path."""

    #: dtype of the residual ring buffers (the model's K/V dtype); the decode
    #: kernel reads bf16 windows.
    kivi_residual_dtype = torch.bfloat16

    # ------------------------------------------------------------------
    # state, geometry, cache binding
    # ------------------------------------------------------------------

    def _init_kivi_state(self, kv_cache_dtype: str | None, vllm_config: Any = None) -> None:
        """All KIVI state; knobs from ``cache_config.kivi_group_size`` /
        ``kivi_residual_length`` (default 128/128), residual rows from
        ``scheduler_config.max_num_seqs`` (attention_backend.py:50-92)."""
        self.enable_kivi = kv_cache_dtype in ("kivi_int4", "kivi")
        cache_config = getattr(vllm_config, "cache_config", None)
        group_size = getattr(cache_config, "kivi_group_size", 128)
        residual_length = getattr(cache_config, "kivi_residual_length", 128)
        self.kivi_group_size = group_size if isinstance(group_size, int) else 128
        self.kivi_residual_length = residual_length if isinstance(residual_length, int) else 128
        if self.enable_kivi:
            self._validate_kivi_geometry()
        self.kivi_bits = 4
        self.k_quant_cache = self.k_scale_cache = self.k_mn_cache = None
        self.v_quant_cache = self.v_scale_cache = self.v_mn_cache = None
        self.kivi_residual_key_cache: torch.Tensor | None = None
        self.kivi_residual_value_cache: torch.Tensor | None = None
        scheduler_config = getattr(vllm_config, "scheduler_config", None)
        max_num_seqs = getattr(scheduler_config, "max_num_seqs", 128)
        self.kivi_max_num_seqs = max_num_seqs if isinstance(max_num_seqs, int) and max_num_seqs > 0 else 128
        self.kivi_residual_req_to_row: dict[str, int] = {}
        self.kivi_residual_row_to_req: list[str | None] = []
        self.kivi_residual_free_rows: list[int] = []
        self._kivi_planner: WindowPlanner | None = None
        self._kivi_plan: tuple[SidePlan, SidePlan] | None = None

    def _validate_kivi_geometry(self) -> None:
        validate_kivi_geometry(
            head_size=self.head_size, group_size=self.kivi_group_size, residual_length=self.kivi_residual_length
        )

    def _check_kivi_cache_bound(self) -> None:
        if any(
            t is None
            for t in (
                self.k_quant_cache, self.k_scale_cache, self.k_mn_cache,
                self.v_quant_cache, self.v_scale_cache, self.v_mn_cache,
            )
        ):
            raise RuntimeError("KIVI cache tensors are not bound.")

    def _get_kivi_block_size(self) -> int:
        self._check_kivi_cache_bound()
        return self.k_quant_cache.shape[-1] * 8

    def _kivi_views(self) -> tuple[torch.Tensor, ...]:
        return (
            self.k_quant_cache, self.k_scale_cache, self.k_mn_cache,
            self.v_quant_cache, self.v_scale_cache, self.v_mn_cache,
        )

    def _bind_kivi_cache(self, kv_cache: Any) -> None:
        """Binds the paged cache: the host's 2 byte buffers become the six
        views (no copy); a 6-tuple is taken as is (attention_backend.py:135-175)."""
        if kv_cache is None:
            return
        if isinstance(kv_cache, torch.Tensor) and kv_cache.dim() == 5 and kv_cache.shape[0] == 2:
            # one host allocation of shape (2, NB, block, KVH, S): its two halves
            kv_cache = (kv_cache[0], kv_cache[1])
        if not isinstance(kv_cache, list | tuple):
            raise RuntimeError(
                "KIVI INT4 kv_cache must be a 2-tuple of byte buffers or a "
                f"6-tuple, got {type(kv_cache)}."
            )
        if len(kv_cache) == 0:
            return
        # the host passes the same buffers every step: bind once
        bound = tuple((t.data_ptr(), tuple(t.shape), t.dtype) if isinstance(t, torch.Tensor) else id(t)
                      for t in kv_cache)
        if bound == getattr(self, "_kivi_bound", None) and self.k_quant_cache is not None:
            return
        if len(kv_cache) == 2:
            kv_cache = kivi_caches_from_byte_tensors(
                *kv_cache,
                layout=kivi_byte_cache_layout(
                    kv_cache[0], kv_cache[1],
                    num_kv_heads=self.num_kv_heads, head_size=self.head_size, group_size=self.kivi_group_size,
                ),
            )
        if len(kv_cache) != 6:
            raise RuntimeError(
                "KIVI INT4 kv_cache must be a 2-tuple of byte buffers or a "
                "6-tuple: (k_quant, k_scale, k_mn, v_quant, v_scale, v_mn)."
            )
        (
            self.k_quant_cache, self.k_scale_cache, self.k_mn_cache,
            self.v_quant_cache, self.v_scale_cache, self.v_mn_cache,
        ) = kv_cache
        self._kivi_bound = bound
        self._ensure_kivi_residual_buffers()

    # ------------------------------------------------------------------
    # residual rows: one per live request (max_num_seqs rows)
    # ------------------------------------------------------------------

    def _ensure_kivi_residual_buffers(self) -> None:
        if self.kivi_residual_key_cache is not None:
            return
        self._check_kivi_cache_bound()
        rows, cap = self.kivi_max_num_seqs, self.kivi_residual_length
        device = self.k_quant_cache.device
        shape = (rows, cap, self.num_kv_heads, self.head_size)
        self.kivi_residual_key_cache = torch.zeros(shape, dtype=self.kivi_residual_dtype, device=device)
        self.kivi_residual_value_cache = torch.zeros(shape, dtype=self.kivi_residual_dtype, device=device)
        self._kivi_planner = WindowPlanner(rows, cap, self.kivi_group_size)
        self.kivi_residual_req_to_row = {}
        self.kivi_residual_row_to_req = [None] * rows
        self.kivi_residual_free_rows = list(range(rows - 1, -1, -1))

    # host views of the per-row FIFO state (same names as the reference)
    @property
    def kivi_residual_key_start(self) -> list[int]:
        self._ensure_kivi_residual_buffers()
        return self._kivi_planner.key.start

    @property
    def kivi_residual_key_len(self) -> list[int]:
        self._ensure_kivi_residual_buffers()
        return self._kivi_planner.key.length

    @property
    def kivi_residual_value_start(self) -> list[int]:
        self._ensure_kivi_residual_buffers()
        return self._kivi_planner.value.start

    @property
    def kivi_residual_value_len(self) -> list[int]:
        self._ensure_kivi_residual_buffers()
        return self._kivi_planner.value.length

    @property
    def kivi_residual_key_slot_ids(self) -> torch.Tensor:
        self._ensure_kivi_residual_buffers()
        return torch.from_numpy(self._kivi_planner.key.slots)

    @property
    def kivi_residual_value_slot_ids(self) -> torch.Tensor:
        self._ensure_kivi_residual_buffers()
        return torch.from_numpy(self._kivi_planner.value.slots)

    def _get_kivi_req_keys(self, req_ids: list[str] | None, num_reqs: int) -> list[str]:
        if req_ids is not None and len(req_ids) >= num_reqs:
            return [str(r) for r in req_ids[:num_reqs]]
        return [f"__kivi_batch_row_{i}" for i in range(num_reqs)]

    def _get_kivi_residual_row(self, req_key: str, *, create: bool) -> int | None:
        self._ensure_kivi_residual_buffers()
        row = self.kivi_residual_req_to_row.get(req_key)
        if row is not None or not create:
            return row
        if not self.kivi_residual_free_rows:
            raise RuntimeError(
                "KIVI residual rows are exhausted. "
                f"max_num_seqs={self.kivi_max_num_seqs}, req_id={req_key}."
            )
        row = self.kivi_residual_free_rows.pop()
        self.kivi_residual_req_to_row[req_key] = row
        self.kivi_residual_row_to_req[row] = req_key
        return row

    def _release_kivi_residual_row(self, req_key: str) -> None:
        row = self.kivi_residual_req_to_row.pop(req_key, None)
        if row is None:
            return
        self._kivi_rows_cache = None
        self.kivi_residual_row_to_req[row] = None
        self._kivi_planner.key.reset(row)
        self._kivi_planner.value.reset(row)
        self.kivi_residual_free_rows.append(row)

    def _release_finished_kivi_residual_rows(self, finished_req_keys: set[str]) -> None:
        for req_key in finished_req_keys:
            self._release_kivi_residual_row(req_key)

    def _get_kivi_residual_lanes(self, row_idx: int, *, is_key: bool) -> list[int]:
        self._ensure_kivi_residual_buffers()
        return self._kivi_planner.side(is_key).lanes(row_idx)

    def _collect_kivi_residual_window(
        self, req_key: str, *, is_key: bool, target_dtype: Any | None = None, target_device: Any | None = None
    ) -> tuple[list[int], torch.Tensor | None]:
        """(slots in FIFO order, window tensors ``[n, KVH, D]``) of a request."""
        row = self._get_kivi_residual_row(req_key, create=False)
        if row is None:
            return [], None
        slots, lanes = self._kivi_planner.window(row, is_key=is_key)
        if not lanes:
            return [], None
        cache = self.kivi_residual_key_cache if is_key else self.kivi_residual_value_cache
        idx = torch.tensor(lanes, dtype=torch.long, device=cache.device)
        tensors = cache[row].index_select(0, idx)
        if target_dtype is not None or target_device is not None:
            tensors = tensors.to(
                device=target_device or tensors.device, dtype=target_dtype or tensors.dtype
            )
        return slots, tensors

    def _has_kivi_residual_entry(self, slot: int, *, req_key: str, is_key: bool) -> bool:
        row = self._get_kivi_residual_row(req_key, create=False)
        if row is None:
            return False
        return bool((self._kivi_planner.side(is_key).slots[row] == int(slot)).any())

    # ------------------------------------------------------------------
    # planned window updates
    # ------------------------------------------------------------------

    def _kivi_begin_plan(self) -> None:
        self._ensure_kivi_residual_buffers()
        self._kivi_plan = self._kivi_planner.begin()
        self._kivi_plan_src: list[torch.Tensor | None] = [None, None]  # new K, new V

    def _kivi_key_flush_gate(self, slots: list[int]) -> None:
        block_size = self._get_kivi_block_size()
        if not is_aligned_key_window(slots, self.kivi_group_size, block_size):
            raise RuntimeError("KIVI key flush requires contiguous aligned token groups.")

    def _kivi_plan_store(self, values: torch.Tensor, slots: list[int], token_index: list[int],
                         *, req_key: str, is_key: bool) -> None:
        row = self._get_kivi_residual_row(req_key, create=True)
        plan = self._kivi_plan[0 if is_key else 1]
        self._kivi_planner.store(plan, row, slots, token_index, is_key=is_key,
                                 gate_block_size=self._get_kivi_block_size() if is_key else 0)

    def _kivi_execute_plan(self) -> None:
        """Applies the open plan: pack every flushed token (one launch per
        side), then land the new tokens and compactions in the ring."""
        if self._kivi_plan is None:
            return
        plans, srcs = self._kivi_plan, self._kivi_plan_src
        self._kivi_plan = None
        exports = [p.export() for p in plans]
        if all(f.size == 0 and w.size == 0 for f, _, w, _ in exports):
            return
        self._launch_kivi_window_apply(exports, srcs)

    def _launch_kivi_window_apply(self, exports, new_tokens) -> None:
        """Device side of a plan (tests may replace it): one upload of the
        plan's index lists, one gather of every flushed and written token (ring
        lanes or new tokens), the pack launches, one scatter into the rings."""
        from ...ops.kivi_window import kivi_window_gather, kivi_window_scatter

        (kfs, kfl, kwl, kws), (vfs, vfl, vwl, vws) = exports
        rk, rv = self.kivi_residual_key_cache, self.kivi_residual_value_cache
        dev = rk.device
        host = np.concatenate([kfs, kws, vfs, vws, kfl, vfl, kwl, vwl])
        idx = torch.from_numpy(host).pin_memory().to(dev, non_blocking=True)
        nfk, nwk, nfv, nwv = kfs.size, kws.size, vfs.size, vws.size
        o = np.cumsum([0, nfk + nwk, nfv + nwv, nfk, nfv, nwk, nwv])
        k_src, v_src = idx[o[0]:o[1]], idx[o[1]:o[2]]
        k_fl, v_fl, k_wl, v_wl = idx[o[2]:o[3]], idx[o[3]:o[4]], idx[o[4]:o[5]], idx[o[5]:o[6]]
        gk, gv = kivi_window_gather(rk, rv, new_tokens[0], new_tokens[1], k_src, v_src)
        if nfk and nfk == nfv and kfl.min() >= 0 and np.array_equal(kfl, vfl):
            # both sides flush the same slots (a bulk prompt write): one launch
            self._write_kivi_kv_quant_cache(gk[:nfk], gv[:nfv], k_fl, kfl.tolist())
        else:
            if nfk:
                self._write_kivi_key_quant_cache(gk[:nfk], k_fl, _host_slots=kfl.tolist())
            if nfv:
                self._write_kivi_value_quant_cache(gv[:nfv], v_fl)
        kivi_window_scatter(rk, rv, k_wl, gk[nfk:], v_wl, gv[nfv:])

    def _kivi_set_plan_source(self, key: torch.Tensor, value: torch.Tensor) -> None:
        dt = self.kivi_residual_dtype
        dev = self.kivi_residual_key_cache.device
        self._kivi_plan_src = [
            key.detach().to(device=dev, dtype=dt).contiguous(),
            value.detach().to(device=dev, dtype=dt).contiguous(),
        ]

    def _store_kivi_residual_entries(self, values: torch.Tensor, slots: torch.Tensor, *, req_key: str,
                                     is_key: bool) -> None:
        """Appends tokens to a request's window, flushing per the asymmetric
        policy (attention_backend.py:411-462); executes immediately."""
        if values.numel() == 0 or slots.numel() == 0:
            return
        self._kivi_begin_plan()
        src = values.detach().to(device=self.kivi_residual_key_cache.device, dtype=self.kivi_residual_dtype)
        self._kivi_plan_src[0 if is_key else 1] = src.contiguous()
        sl = _host_list(slots)
        self._kivi_plan_store(src, sl, list(range(len(sl))), req_key=req_key, is_key=is_key)
        self._kivi_execute_plan()

    def _write_kivi_cache(self, key: Any, value: Any, slot_mapping: Any, req_ids: list[str] | None,
                          actual_seq_qlen: Any) -> None:
        """Incremental write of every request's new tokens through its window
        (attention_backend.py:562-606), planned once for the whole batch."""
        if key is None or value is None or slot_mapping is None:
            return
        qlen = _host_list(actual_seq_qlen)
        if not qlen:
            return
        slots_all = _host_list(slot_mapping)
        keys = self._get_kivi_req_keys(req_ids, len(qlen))
        self._kivi_begin_plan()
        self._kivi_set_plan_source(key, value)
        n = len(slots_all)
        if len(qlen) == n and qlen == list(range(1, n + 1)) and min(slots_all) >= 0:
            # decode step: one token per request, planned for the whole batch
            rows = [self._get_kivi_residual_row(k, create=True) for k in keys[:n]]
            tok = list(range(n))
            self._kivi_planner.store_one_each(self._kivi_plan[0], rows, slots_all, tok, is_key=True,
                                              gate_block_size=self._get_kivi_block_size())
            self._kivi_planner.store_one_each(self._kivi_plan[1], rows, slots_all, tok, is_key=False)
            self._kivi_execute_plan()
            return
        prev = 0
        for r, q_end in enumerate(qlen):
            q_end = min(int(q_end), n)
            if prev >= n:
                break
            if q_end <= prev:
                prev = q_end
                continue
            idx = [i for i in range(prev, q_end) if slots_all[i] >= 0]
            if idx:
                sl = [slots_all[i] for i in idx]
                self._kivi_plan_store(None, sl, idx, req_key=keys[r], is_key=True)
                self._kivi_plan_store(None, sl, idx, req_key=keys[r], is_key=False)
            prev = q_end
        self._kivi_execute_plan()

    def _write_kivi_prefill_cache(self, key: Any, value: Any, slot_mapping: Any, req_ids: list[str] | None,
                                  actual_seq_qlen: Any) -> None:
        """Bulk prompt write (attention_backend.py:608-674): the first
        floor(n / r) * r tokens go straight to the int4 history, the rest to
        the window."""
        if key is None or value is None or slot_mapping is None:
            return
        qlen = _host_list(actual_seq_qlen)
        if not qlen:
            return
        slots_all = _host_list(slot_mapping)
        keys = self._get_kivi_req_keys(req_ids, len(qlen))
        r_len = self.kivi_residual_length
        self._kivi_begin_plan()
        self._kivi_set_plan_source(key, value)
        kplan, vplan = self._kivi_plan
        n = len(slots_all)
        prev = 0
        for r, q_end in enumerate(qlen):
            q_end = min(int(q_end), n)
            if prev >= n:
                break
            if q_end <= prev:
                prev = q_end
                continue
            idx = [i for i in range(prev, q_end) if slots_all[i] >= 0]
            if not idx:
                prev = q_end
                continue
            sl = [slots_all[i] for i in idx]
            flush = (len(idx) // r_len) * r_len
            if flush:
                self._kivi_key_flush_gate(sl[:flush])
                self._kivi_planner.flush_direct(kplan, sl[:flush], idx[:flush])
                self._kivi_planner.flush_direct(vplan, sl[:flush], idx[:flush])
            if flush < len(idx):
                self._kivi_plan_store(None, sl[flush:], idx[flush:], req_key=keys[r], is_key=True)
                self._kivi_plan_store(None, sl[flush:], idx[flush:], req_key=keys[r], is_key=False)
            prev = q_end
        self._kivi_execute_plan()

    def _write_kivi_key_quant_cache(self, key: Any, slot_mapping: Any, _host_slots: list[int] | None = None) -> None:
        """Whole-group key flush into the int4 history with every layout check
        before the launch (attention_backend.py:676-726)."""
        self._check_kivi_cache_bound()
        if key is None or slot_mapping is None:
            return
        host_slots = _host_slots if _host_slots is not None else _host_list(slot_mapping)
        keep = [i for i, s in enumerate(host_slots) if s >= 0]
        if not keep:
            return
        if len(keep) != len(host_slots):
            sel = torch.tensor(keep, dtype=torch.long, device=key.device)
            key = key.index_select(0, sel)
            slot_mapping = slot_mapping.index_select(0, sel.to(slot_mapping.device))
            host_slots = [host_slots[i] for i in keep]
        key = key.contiguous()
        slots = slot_mapping.to(torch.long).contiguous()
        if key.shape[-1] != self.head_size:
            raise RuntimeError(
                f"KIVI INT4 key head_size must match attention head_size ({self.head_size}), got {key.shape[-1]}."
            )
        if key.shape[0] % self.kivi_group_size != 0:
            raise RuntimeError(
                "KIVI key flush must contain whole token groups, got "
                f"{key.shape[0]} tokens for group_size={self.kivi_group_size}."
            )
        if self.head_size % 8 != 0:
            raise RuntimeError(
                f"KIVI INT4 int32 packing requires head_size ({self.head_size}) to be divisible by 8."
            )
        if self.kivi_group_size % 8 != 0:
            raise RuntimeError(
                f"KIVI INT4 key packing requires kivi_group_size ({self.kivi_group_size}) to be divisible by 8."
            )
        block_size = self._get_kivi_block_size()
        if block_size % self.kivi_group_size != 0:
            raise RuntimeError(
                f"KIVI INT4 key cache requires block_size ({block_size}) to be "
                f"divisible by kivi_group_size ({self.kivi_group_size})."
            )
        if not is_aligned_key_window(host_slots, self.kivi_group_size, block_size):
            raise RuntimeError("KIVI key flush requires contiguous aligned token groups.")
        self._launch_kivi_key_pack(key, slots)

    def _write_kivi_kv_quant_cache(self, key: Any, value: Any, slot_mapping: Any, host_slots: list[int]) -> None:
        """Key and value flush of the same (valid) slots, with both sides'
        checks before the one launch (qkv_kivi_pack_kv)."""
        self._check_kivi_cache_bound()
        block_size = self._get_kivi_block_size()
        g = self.kivi_group_size
        if key.shape[-1] != self.head_size or value.shape[-1] != self.head_size:
            raise RuntimeError(
                f"KIVI INT4 key/value head_size must match attention head_size ({self.head_size})."
            )
        if key.shape[0] % g != 0:
            raise RuntimeError(
                f"KIVI key flush must contain whole token groups, got {key.shape[0]} tokens for group_size={g}."
            )
        if self.head_size % 8 != 0 or g % 8 != 0 or self.head_size % g != 0 or block_size % g != 0:
            raise RuntimeError("KIVI INT4 packing geometry is invalid for this cache.")
        if not is_aligned_key_window(host_slots, g, block_size):
            raise RuntimeError("KIVI key flush requires contiguous aligned token groups.")
        self._launch_kivi_kv_pack(key.contiguous(), value.contiguous(), slot_mapping.to(torch.long).contiguous())

    def _launch_kivi_kv_pack(self, key: Any, value: Any, slots: Any) -> None:
        """Kernel launch seam of the two-sided flush."""
        from ...ops.kivi_pack import kivi_pack_kv_cache

        kivi_pack_kv_cache(
            key, value, slots, (self.k_quant_cache, self.k_scale_cache, self.k_mn_cache),
            (self.v_quant_cache, self.v_scale_cache, self.v_mn_cache), self.kivi_group_size, validate_slots=False,
        )

    def _launch_kivi_key_pack(self, key: Any, slots: Any) -> None:
        """Kernel launch seam (tests may replace it)."""
        from ...ops.kivi_pack import kivi_pack_key_cache

        kivi_pack_key_cache(
            key, slots, self.k_quant_cache, self.k_scale_cache, self.k_mn_cache, self.kivi_group_size,
            validate_slots=False,
        )

    def _write_kivi_value_quant_cache(self, value: Any, slot_mapping: Any) -> None:
        """Value pack with the reference's checks (attention_backend.py:741-777)."""
        self._check_kivi_cache_bound()
        if value is None or slot_mapping is None:
            return
        head_size = value.shape[-1]
        if head_size != self.head_size:
            raise RuntimeError(
                f"KIVI INT4 value head_size must match attention head_size ({self.head_size}), got {head_size}."
            )
        if head_size % self.kivi_group_size != 0:
            raise RuntimeError(
                f"KIVI INT4 value head_size ({head_size}) must be divisible by "
                f"kivi_group_size ({self.kivi_group_size})."
            )
        if head_size % 8 != 0:
            raise RuntimeError(f"KIVI INT4 int32 packing requires head_size ({head_size}) to be divisible by 8.")
        if self.kivi_group_size % 8 != 0:
            raise RuntimeError(
                f"KIVI INT4 value packing requires kivi_group_size ({self.kivi_group_size}) to be divisible by 8."
            )
        # negative slots are skipped by the kernel itself
        self._launch_kivi_value_pack(value.contiguous(), slot_mapping.to(torch.long).contiguous())

    def _launch_kivi_value_pack(self, value: Any, slots: Any) -> None:
        """Kernel launch seam (tests may replace it)."""
        from ...ops.kivi_pack import kivi_pack_value_cache

        kivi_pack_value_cache(
            value, slots, self.v_quant_cache, self.v_scale_cache, self.v_mn_cache, self.kivi_group_size
        )

    # ------------------------------------------------------------------
    # window sync
    # ------------------------------------------------------------------

    def _sync_kivi_residual_windows(self, block_table: Any, seq_lens: list[int], req_ids: list[str] | None,
                                    finished_req_ids: set[str] | None = None) -> None:
        """Releases finished rows and drops window slots a request no longer
        owns (attention_backend.py:813-836). The common case — both windows
        hold exactly the last positions — is checked in O(window); only a
        mismatch expands the request's full slot list."""
        if finished_req_ids:
            self._release_finished_kivi_residual_rows({str(r) for r in finished_req_ids})
        keys = self._get_kivi_req_keys(req_ids, len(seq_lens))
        rows = [(i, self.kivi_residual_req_to_row.get(k)) for i, k in enumerate(keys)]
        rows = [(i, r) for i, r in rows if r is not None]
        if not rows:
            return
        bt = block_table
        if isinstance(bt, torch.Tensor):
            bt = (bt.cpu() if bt.is_cuda else bt).numpy()
        bt = np.asarray(bt)
        block_size = self._get_kivi_block_size()
        planner = self._kivi_planner
        idx = np.fromiter((i for i, _ in rows), dtype=np.int64, count=len(rows))
        rws = np.fromiter((r for _, r in rows), dtype=np.int64, count=len(rows))
        live = planner.expected_live_rows(rws, np.asarray(seq_lens, dtype=np.int64)[idx], bt[idx], block_size)
        stale = [rows[j] for j in np.flatnonzero(~live)]
        if not stale:
            return
        own_plan = self._kivi_plan is None
        if own_plan:
            self._kivi_begin_plan()
        for i, r in stale:
            live = set(ordered_slots(bt[i:i + 1], [int(seq_lens[i])], block_size)[0])
            planner.prune(self._kivi_plan[0], r, live, is_key=True)
            planner.prune(self._kivi_plan[1], r, live, is_key=False)
        if own_plan:
            self._kivi_execute_plan()

    # ------------------------------------------------------------------
    # attention
    # ------------------------------------------------------------------

    def _is_kivi_chunked_prefill_all_new(self, attn_metadata: Any) -> bool:
        qlen = attn_metadata.actual_seq_lengths_q
        nd = attn_metadata.num_decodes
        for i in range(nd, len(attn_metadata.seq_lens_list)):
            q_start = qlen[i - 1] if i > 0 else 0
            if attn_metadata.seq_lens_list[i] > qlen[i] - q_start:
                return False
        return True

    def forward(self, layer: Any, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, kv_cache: Any,
                attn_metadata: Any, output: torch.Tensor | None = None, output_scale: torch.Tensor | None = None,
                output_block_scale: torch.Tensor | None = None) -> torch.Tensor:
        """INT4 forward entry (attention_backend.py:972-1004); bypasses the
        host's reshape_and_cache."""
        assert output is not None, "Output tensor must be provided."
        if not getattr(self, "enable_kivi", False):
            raise RuntimeError(
                "the KIVI INT4 attention impl was instantiated without the "
                "kivi_int4 cache dtype; check the host get_impl_cls dispatch"
            )
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError(
                "fused output quantization is not yet supported for AscendKiviInt4AttentionBackendImpl"
            )
        if attn_metadata is None:
            return output.fill_(0)
        return self._forward_kivi_attention(query, key, value, attn_metadata, output, kv_cache)

    def _forward_kivi_attention(self, query, key, value, attn_metadata, output, kv_cache=None):
        """Dispatch by attention state (attention_backend.py:1006-1191)."""
        self._bind_kivi_cache(kv_cache)
        finished = getattr(attn_metadata, "finished_req_ids", None)
        if finished:
            self._release_finished_kivi_residual_rows({str(r) for r in finished})
        state = _attn_state_name(attn_metadata)
        seq_lens = _host_list(attn_metadata.seq_lens_list)
        req_ids = getattr(attn_metadata, "req_ids", None)
        if state == "DecodeOnly":
            qlen = list(range(1, len(seq_lens) + 1))
        else:
            qlen = _host_list(attn_metadata.actual_seq_lengths_q)
        num_tokens = int(qlen[-1])
        query = query[:num_tokens]

        if state == "PrefillNoCache":
            if key is None or value is None:
                raise RuntimeError("KIVI PrefillNoCache requires dense key/value.")
            n = min(getattr(attn_metadata, "num_actual_tokens", key.shape[0]), key.shape[0])
            self._write_kivi_prefill_cache(key[:n], value[:n], attn_metadata.slot_mapping[:n], req_ids, qlen)
            return self._forward_kivi_prefill_fia(query, key, value, attn_metadata, output)

        history = state == "ChunkedPrefill" and not self._is_kivi_chunked_prefill_all_new(attn_metadata)

        if state == "DecodeOnly":
            if key is not None and value is not None and self._kivi_native_decode(
                    query, key, value, attn_metadata, seq_lens, req_ids, output):
                return output
            if key is not None and value is not None:
                n = min(getattr(attn_metadata, "num_actual_tokens", key.shape[0]), key.shape[0])
                if n > 0:
                    self._write_kivi_cache(key[:n], value[:n], attn_metadata.slot_mapping[:n], req_ids,
                                           list(range(1, len(seq_lens) + 1)))
            self._sync_kivi_residual_windows(attn_metadata.block_tables, seq_lens, req_ids, finished)
            return self._forward_kivi_paged_decode_attention(query, attn_metadata.block_tables, seq_lens,
                                                             req_ids, output)

        if state == "ChunkedPrefill" and not history:
            if key is not None and value is not None:
                n = min(getattr(attn_metadata, "num_actual_tokens", key.shape[0]), key.shape[0])
                if n > 0:
                    nd_tok = min(attn_metadata.num_decode_tokens, n)
                    nd = attn_metadata.num_decodes
                    slot_mapping = attn_metadata.slot_mapping[:n]
                    if nd_tok > 0:
                        self._write_kivi_cache(key[:nd_tok], value[:nd_tok], slot_mapping[:nd_tok],
                                               None if req_ids is None else req_ids[:nd],
                                               list(range(1, nd + 1)))
                    if nd_tok < n:
                        pre_q = [int(qlen[i]) - nd_tok for i in range(nd, len(qlen))]
                        self._write_kivi_prefill_cache(key[nd_tok:n], value[nd_tok:n], slot_mapping[nd_tok:n],
                                                       None if req_ids is None else req_ids[nd:], pre_q)
            self._sync_kivi_residual_windows(attn_metadata.block_tables, seq_lens, req_ids, finished)
            return self._forward_kivi_chunked_prefill(query, key, value, attn_metadata, output)

        # every other state (and chunked prefill with history): incremental
        # write of all rows, sync, attention over history + window
        if key is not None and value is not None:
            n = min(getattr(attn_metadata, "num_actual_tokens", key.shape[0]), key.shape[0])
            if n > 0:
                self._write_kivi_cache(key[:n], value[:n], attn_metadata.slot_mapping[:n], req_ids, qlen)
        self._sync_kivi_residual_windows(attn_metadata.block_tables, seq_lens, req_ids, finished)
        causal = bool(getattr(attn_metadata, "causal", True))
        return self._forward_kivi_history_attention(query, attn_metadata.block_tables, seq_lens, qlen, req_ids,
                                                    causal, output)

    # -- kernel calls ---------------------------------------------------

    def _kivi_native_decode(self, query, key, value, attn_metadata, seq_lens, req_ids, output) -> bool:
        """The whole DecodeOnly step (window writes, window sync, decode
        attention) as one native call, ``qkv_kivi_decode_step``; False when
        the batch is not one new token per request with valid slots (the
        general path then runs)."""
        from ...ops.kivi_step import KiviDecodeStep

        B = len(seq_lens)
        n = min(getattr(attn_metadata, "num_actual_tokens", key.shape[0]), key.shape[0])
        if B == 0 or n != B or self.kivi_residual_dtype != torch.bfloat16 or query.shape[0] < B:
            return False
        slots = _host_i64(attn_metadata.slot_mapping, B)
        if slots.size != B or slots.min() < 0:
            return False
        self._ensure_kivi_residual_buffers()
        rows = self._kivi_rows_of(self._get_kivi_req_keys(req_ids, B))
        bt = attn_metadata.block_tables
        bt_dev = None  # a host table is staged by the step with its indices
        if isinstance(bt, torch.Tensor):
            if bt.is_cuda:
                bt_dev = self._kivi_table(bt, B)
                bt_host = bt[:B].cpu().numpy()
            else:
                bt_host = bt[:B].numpy()
        else:
            bt_host = np.asarray(bt)[:B]
        if bt_host.dtype != np.int32 or not bt_host.flags.c_contiguous:
            bt_host = np.ascontiguousarray(bt_host, dtype=np.int32)
        dev = self.kivi_residual_key_cache.device
        k = key[:B] if key.dtype == torch.bfloat16 and key.device == dev else key[:B].to(dev, torch.bfloat16)
        v = value[:B] if value.dtype == torch.bfloat16 and value.device == dev else value[:B].to(dev, torch.bfloat16)
        step = getattr(self, "_kivi_step", None)
        if step is None:
            step = self._kivi_step = KiviDecodeStep()
        if getattr(self, "_kivi_step_bound", None) is not self._kivi_bound:
            step.bind(self._kivi_planner._handle, self._kivi_views(), self.kivi_residual_key_cache,
                      self.kivi_residual_value_cache, self.kivi_group_size, self.scale)
            self._kivi_step_bound = self._kivi_bound
        step.run(rows, slots, np.asarray(seq_lens, dtype=np.int32), bt_host, bt_dev, query[:B], k.contiguous(),
                 v.contiguous(), output[:B])
        return True

    def _kivi_rows_of(self, keys: list[str]) -> np.ndarray:
        """Residual rows of the batch's requests (created on first sight),
        reused while the batch's request list and the row map are unchanged."""
        cached = getattr(self, "_kivi_rows_cache", None)
        if cached is not None and cached[0] == keys:
            return cached[1]
        rows = np.fromiter((self._get_kivi_residual_row(k, create=True) for k in keys), dtype=np.int64,
                           count=len(keys))
        self._kivi_rows_cache = (keys, rows)
        return rows

    def _kivi_res_state(self, req_keys: list[str], ends: list[int]) -> np.ndarray:
        st = np.zeros((len(req_keys), 6), dtype=np.int32)
        st[:, 0] = -1
        planner = self._kivi_planner
        for i, k in enumerate(req_keys):
            row = self.kivi_residual_req_to_row.get(k)
            st[i, 5] = ends[i]
            if row is None:
                continue
            st[i, 0] = row
            st[i, 1] = planner.key.start[row]
            st[i, 2] = planner.key.length[row]
            st[i, 3] = planner.value.start[row]
            st[i, 4] = planner.value.length[row]
        return st

    def _kivi_device_i32(self, arr) -> torch.Tensor:
        t = torch.from_numpy(np.ascontiguousarray(arr, dtype=np.int32))
        return t.to(self.k_quant_cache.device, non_blocking=True)

    def _kivi_table(self, block_table: Any, rows: int) -> torch.Tensor:
        """The first ``rows`` block-table rows as int32 on the device. A host
        table lands in a buffer this layer reuses: the result is valid until
        the next call (kernels enqueued before it on the stream are safe)."""
        dev = self.k_quant_cache.device
        if isinstance(block_table, torch.Tensor):
            bt = block_table[:rows]
            if bt.device == dev:
                return bt.to(torch.int32).contiguous()
            # a host table: one copy into a device buffer kept for the shape
            buf = getattr(self, "_kivi_bt_dev", None)
            if buf is None or buf.shape != bt.shape:
                buf = self._kivi_bt_dev = torch.empty(bt.shape, dtype=torch.int32, device=dev)
            buf.copy_(bt, non_blocking=True)
            return buf
        return self._kivi_device_i32(np.asarray(block_table)[:rows])

    def _forward_kivi_paged_decode_attention(self, query, block_table, seq_lens, req_ids, output):
        """One query token per request over int4 pages + window
        (replaces attention_backend.py:1193-1230)."""
        from ...ops.kivi_decode import kivi_paged_decode

        B = len(seq_lens)
        if B == 0:
            return output
        self._ensure_kivi_residual_buffers()
        keys = self._get_kivi_req_keys(req_ids, B)
        res_state = self._kivi_device_i32(self._kivi_res_state(keys, list(seq_lens)))
        sl = self._kivi_device_i32(seq_lens)
        bt = self._kivi_table(block_table, B)
        kivi_paged_decode(
            query[:B], self._kivi_views(), self.kivi_residual_key_cache, self.kivi_residual_value_cache,
            bt, sl, res_state, self.kivi_group_size, self.scale, output[:B], max(seq_lens),
        )
        return output

    def _forward_kivi_history_attention(self, query, block_table, seq_lens, qlen, req_ids, causal, output):
        """Rows over history + window (the reference's generic branch,
        attention_backend.py:1176-1191). Requests with several query tokens
        (prefill chunks on cached tokens) gather their K/V densely (int4 pages
        dequantised + bf16 window) and run the tensor-core prompt attention,
        aligned to the end of their keys; single-token rows run the paged
        decode kernel, each with its causal length."""
        from ...ops.kivi_decode import kivi_paged_decode
        from ..history_rows import RowView, dense_prefill_geometry_ok, plan_history_rows

        B = len(seq_lens)
        plan = plan_history_rows(qlen[:B], seq_lens, causal,
                                 dense_prefill_geometry_ok(self.head_size, self.num_heads, self.num_kv_heads))
        if plan.num_tokens == 0:
            return output
        keys = self._get_kivi_req_keys(req_ids, B)
        self._ensure_kivi_residual_buffers()
        st_all = self._kivi_res_state(keys, plan.seq_lens)
        bt_full = self._kivi_table(block_table, B)
        if plan.dense:
            self._kivi_dense_history(query, bt_full, st_all, plan, causal, output)
        if not plan.rows_req:
            return output
        sel = torch.tensor(plan.rows_req, dtype=torch.long).to(bt_full.device, non_blocking=True)
        rows = RowView(query, output, plan.rows_q)
        kivi_paged_decode(
            rows.query, self._kivi_views(), self.kivi_residual_key_cache, self.kivi_residual_value_cache,
            bt_full.index_select(0, sel).contiguous(), self._kivi_device_i32(plan.rows_len),
            self._kivi_device_i32(st_all[plan.rows_req]), self.kivi_group_size, self.scale, rows.output,
            max(max(plan.rows_len), 1),
        )
        rows.commit()
        return output

    def _kivi_dense_history(self, query, bt_full, st_all, plan, causal, output):
        """Dense chunks of ``plan``: one gather of their K/V (int4 history +
        window) and one prompt-attention launch over all of them."""
        from ...ops.kivi_gather import kivi_dequant_gather
        from ...ops.prefill import dense_prefill
        from ..history_rows import RowView

        reqs = plan.dense
        sel = torch.tensor(reqs, dtype=torch.long).to(bt_full.device, non_blocking=True)
        kv_lens = [plan.seq_lens[b] for b in reqs]
        dk, dv = kivi_dequant_gather(self._kivi_views(), self.kivi_residual_key_cache,
                                     self.kivi_residual_value_cache, bt_full.index_select(0, sel).contiguous(),
                                     kv_lens, self._kivi_device_i32(st_all[reqs]), self.kivi_group_size)
        rows = RowView(query, output, [plan.starts[b] + i for b in reqs for i in range(plan.q_lens[b])])
        dense_prefill(rows.query.contiguous(), dk, dv, [plan.q_lens[b] for b in reqs], kv_lens, self.scale,
                      rows.output, causal=causal)
        rows.commit()

    def _forward_kivi_prefill_fia(self, query, key, value, attn_metadata, output):
        """Causal prompt attention over the raw prompt K/V
        (replaces attention_backend.py:1232-1266)."""
        from ...ops.prefill import dense_prefill

        qlen = _host_list(attn_metadata.actual_seq_lengths_q)
        n = int(qlen[-1])
        lens = [qlen[0]] + [qlen[i] - qlen[i - 1] for i in range(1, len(qlen))]
        dense_prefill(query[:n].contiguous(), key[:n].contiguous(), value[:n].contiguous(), lens, lens,
                      self.scale, output[:n], causal=bool(attn_metadata.causal))
        return output

    def _forward_kivi_chunked_prefill(self, query, key, value, attn_metadata, output):
        """Decode rows over the paged history, all-new prompt rows over their
        own raw K/V (replaces attention_backend.py:1268-1339)."""
        from ...ops.prefill import dense_prefill

        nd_tok = attn_metadata.num_decode_tokens
        nd = attn_metadata.num_decodes
        qlen = _host_list(attn_metadata.actual_seq_lengths_q)
        seq_lens = _host_list(attn_metadata.seq_lens_list)
        num_tokens = int(qlen[-1])
        req_ids = getattr(attn_metadata, "req_ids", None)
        if nd_tok > 0:
            self._forward_kivi_paged_decode_attention(
                query[:nd_tok], attn_metadata.block_tables[:nd], seq_lens[:nd],
                None if req_ids is None else req_ids[:nd], output,
            )
        if attn_metadata.num_prefills <= 0:
            return output
        if key is None or value is None:
            raise RuntimeError("KIVI ChunkedPrefill requires dense key/value for all-new prefill prompts.")
        pre_q = [qlen[i] - nd_tok for i in range(nd, len(qlen))]
        lens = [pre_q[0]] + [pre_q[i] - pre_q[i - 1] for i in range(1, len(pre_q))]
        out = output[nd_tok:num_tokens]
        dense_prefill(query[nd_tok:num_tokens].contiguous(), key[nd_tok:num_tokens].contiguous(),
                      value[nd_tok:num_tokens].contiguous(), lens, lens, self.scale, out,
                      causal=bool(attn_metadata.causal))
        return output


__all__ = ["AscendKiviInt4AttentionBackendMixin"]
