"""FP8 per-token-head attention implementation for B200 (plugin mixin).

The reference ships this method's contract, byte layout, CPU semantics and
store kernel (methods/fp8_per_token_head/, ops/triton/per_token_head_store.py)
but no read path and no adapter. This mixin is that read path, shaped like the
INT8 mixin: every forward quantises its new K/V into the pages
(``qkv_fp8_store``: E4M3 + one fp32 scale per (token, head)), then attends by
state:

* DecodeOnly: ``qkv_fp8_paged_decode`` over the pages;
* PrefillNoCache / all-new prompts: prompt attention over the raw K/V;
* chunks over cached keys: the FP8 dense gather + tensor-core prompt
  attention (aligned to the end of the keys); single-token rows: the paged
  decode kernel with their causal length.
"""

from __future__ import annotations

from typing import Any

import numpy as np
import torch

from .byte_cache import fp8_caches_from_byte_tensors, fp8_per_token_head_layout


def _state_name(attn_metadata: Any) -> str:
    state = getattr(attn_metadata, "attn_state", None)
    return getattr(state, "name", str(state))


def _host_list(x) -> list[int]:
    if isinstance(x, torch.Tensor):
        return [int(v) for v in x.tolist()]
    return [int(v) for v in x]


class AscendFp8PerTokenHeadAttentionBackendMixin:
    """Per-token-head E4M3 KV cache on the B200 kernels."""

    k_data: torch.Tensor | None = None
    k_scale: torch.Tensor | None = None
    v_data: torch.Tensor | None = None
    v_scale: torch.Tensor | None = None

    def forward(self, layer: Any, query: torch.Tensor, key: torch.Tensor | None, value: torch.Tensor | None,
                kv_cache: Any, attn_metadata: Any, output: torch.Tensor | None = None,
                output_scale: torch.Tensor | None = None,
                output_block_scale: torch.Tensor | None = None) -> torch.Tensor:
        assert output is not None, "Output tensor must be provided."
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError(
                "fused output quantization is not yet supported for AscendFp8PerTokenHeadAttentionBackendImpl"
            )
        if attn_metadata is None:
            return output.fill_(0)
        self._bind_fp8_cache(kv_cache)
        state = _state_name(attn_metadata)
        if key is not None and value is not None:
            n = min(int(getattr(attn_metadata, "num_actual_tokens", key.shape[0])), key.shape[0])
            if n > 0:
                self._store_fp8(key[:n], value[:n], attn_metadata.slot_mapping[:n])
        if state == "DecodeOnly":
            seq_lens = _host_list(attn_metadata.seq_lens_list)
            return self._fp8_paged(query, attn_metadata.block_tables, seq_lens, output)
        qlen = _host_list(attn_metadata.actual_seq_lengths_q)
        seq_lens = _host_list(attn_metadata.seq_lens_list)
        if state == "ChunkedPrefill":
            return self._forward_fp8_chunked(query, key, value, attn_metadata, qlen, seq_lens, output)
        lens = [qlen[0]] + [qlen[i] - qlen[i - 1] for i in range(1, len(qlen))]
        if state == "PrefillNoCache" and key is not None and all(s <= q for s, q in zip(seq_lens, lens)):
            return self._fp8_dense(query, key, value, lens, output, causal=bool(getattr(attn_metadata, "causal", True)))
        return self._fp8_history(query, attn_metadata.block_tables, seq_lens, qlen, output,
                                 causal=bool(getattr(attn_metadata, "causal", True)))

    # -- cache ------------------------------------------------------------

    def _bind_fp8_cache(self, kv_cache: Any) -> None:
        """The host's two byte buffers (or one (2, NB, block, KVH, S) tensor)
        become the four views (no copy); a 4-tuple is taken as is."""
        if kv_cache is None:
            return
        if isinstance(kv_cache, torch.Tensor) and kv_cache.dim() == 5 and kv_cache.shape[0] == 2:
            kv_cache = (kv_cache[0], kv_cache[1])
        if not isinstance(kv_cache, list | tuple) or len(kv_cache) not in (2, 4):
            raise RuntimeError(
                "fp8_per_token_head kv_cache must be a 2-tuple of byte buffers or a 4-tuple "
                "(k_data, k_scale, v_data, v_scale)."
            )
        bound = tuple((t.data_ptr(), tuple(t.shape), t.dtype) for t in kv_cache)
        if bound == getattr(self, "_fp8_bound", None):
            return
        if len(kv_cache) == 2:
            lay = fp8_per_token_head_layout(kv_cache[0], kv_cache[1], num_kv_heads=self.num_kv_heads,
                                            head_size=self.head_size)
            kv_cache = fp8_caches_from_byte_tensors(kv_cache[0], kv_cache[1], lay)
        self.k_data, self.k_scale, self.v_data, self.v_scale = kv_cache
        self._fp8_bound = bound

    def _fp8_views(self):
        if self.k_data is None:
            raise RuntimeError("fp8_per_token_head KV cache tensors are not bound.")
        return self.k_data, self.k_scale, self.v_data, self.v_scale

    def _store_fp8(self, key, value, slot_mapping) -> None:
        """Quantise + scatter (the store contract of
        ops/triton/per_token_head_store.py:262-294)."""
        from ...ops.fp8 import fp8_store

        fp8_store(key, value, slot_mapping, *self._fp8_views())

    # -- attention --------------------------------------------------------

    def _fp8_device_i32(self, arr) -> torch.Tensor:
        t = torch.from_numpy(np.ascontiguousarray(arr, dtype=np.int32))
        return t.to(self.k_data.device, non_blocking=True)

    def _fp8_table(self, block_table, rows: int) -> torch.Tensor:
        dev = self.k_data.device
        if isinstance(block_table, torch.Tensor):
            bt = block_table[:rows]
            if bt.device != dev:
                bt = bt.to(dev, non_blocking=True)
            return bt.to(torch.int32).contiguous()
        return self._fp8_device_i32(np.asarray(block_table)[:rows])

    def _fp8_paged(self, query, block_table, seq_lens, output, rows_req=None):
        """Decode rows: query row i over ``seq_lens[i]`` keys of request
        ``rows_req[i]`` (row i itself when ``rows_req`` is None)."""
        from ...ops.fp8 import fp8_paged_decode

        B = len(seq_lens)
        if B == 0:
            return output
        bt = self._fp8_table(block_table, (max(rows_req) + 1) if rows_req else B)
        if rows_req is not None:
            sel = torch.tensor(rows_req, dtype=torch.long).to(bt.device, non_blocking=True)
            bt = bt.index_select(0, sel).contiguous()
        fp8_paged_decode(query[:B], *self._fp8_views(), bt, self._fp8_device_i32(seq_lens), self.scale, output[:B],
                         max(max(seq_lens), 1))
        return output

    def _fp8_dense(self, query, key, value, lens, output, causal=True):
        from ...ops.prefill import dense_prefill

        n = sum(lens)
        dense_prefill(query[:n].contiguous(), key[:n].contiguous(), value[:n].contiguous(), lens, lens, self.scale,
                      output[:n], causal=causal)
        return output

    def _fp8_history(self, query, block_table, seq_lens, qlen, output, causal=True):
        """Rows over the pages: multi-token requests gather dense K/V and run
        the tensor-core prompt attention; single rows the paged decode."""
        from ...ops.fp8 import fp8_dequant_gather
        from ...ops.prefill import dense_prefill
        from ..history_rows import RowView, dense_prefill_geometry_ok, plan_history_rows

        B = len(qlen)
        plan = plan_history_rows(qlen, seq_lens[:B], causal,
                                 dense_prefill_geometry_ok(self.head_size, self.num_heads, self.num_kv_heads))
        if plan.num_tokens == 0:
            return output
        if plan.dense:
            reqs = plan.dense
            bt = self._fp8_table(block_table, max(reqs) + 1)
            sel = torch.tensor(reqs, dtype=torch.long).to(bt.device, non_blocking=True)
            kv_lens = [plan.seq_lens[b] for b in reqs]
            dk, dv = fp8_dequant_gather(*self._fp8_views(), bt.index_select(0, sel).contiguous(), kv_lens)
            rows = RowView(query, output, [plan.starts[b] + i for b in reqs for i in range(plan.q_lens[b])])
            dense_prefill(rows.query.contiguous(), dk, dv, [plan.q_lens[b] for b in reqs], kv_lens, self.scale,
                          rows.output, causal=causal)
            rows.commit()
        if plan.rows_req:
            rows = RowView(query, output, plan.rows_q)
            self._fp8_paged(rows.query, block_table, plan.rows_len, rows.output, rows_req=plan.rows_req)
            rows.commit()
        return output

    def _forward_fp8_chunked(self, query, key, value, attn_metadata, qlen, seq_lens, output):
        """Decode rows first (one token each), then the prompt rows: over the
        raw K/V when every prompt is new, else over the pages."""
        nd_tok = int(getattr(attn_metadata, "num_decode_tokens", 0))
        nd = int(getattr(attn_metadata, "num_decodes", 0))
        num_tokens = int(qlen[-1])
        if nd_tok > 0:
            self._fp8_paged(query, attn_metadata.block_tables[:nd], seq_lens[:nd], output)
        if int(getattr(attn_metadata, "num_prefills", len(qlen) - nd)) <= 0:
            return output
        pre_q = [qlen[i] - nd_tok for i in range(nd, len(qlen))]
        lens = [pre_q[0]] + [pre_q[i] - pre_q[i - 1] for i in range(1, len(pre_q))]
        sub_q, sub_o = query[nd_tok:num_tokens], output[nd_tok:num_tokens]
        if key is not None and all(seq_lens[nd + i] <= lens[i] for i in range(len(lens))):
            return self._fp8_dense(sub_q, key[nd_tok:num_tokens], value[nd_tok:num_tokens], lens, sub_o) and output
        self._fp8_history(sub_q, attn_metadata.block_tables[nd:], seq_lens[nd:], pre_q, sub_o)
        return output


__all__ = ["AscendFp8PerTokenHeadAttentionBackendMixin"]
