"""Dynamic per-channel INT8 attention implementation for B200 (plugin mixin).

Same role and method names as the reference's ``AscendInt8AttentionBackendMixin``
(methods/int8_dynamic/attention_backend.py of vllm_ascend_quantized_kv_cache):
per-layer scales calibrated once from the first K/V a layer sees, quantised
writes into the int8 pages, and attention by state:

* DecodeOnly: ``qkv_int8_paged_decode`` (replaces the FIA BNSD call, :173-205);
* ChunkedPrefill: decode rows as above; prompt rows over their raw K/V when all
  prompts are new, else over the int8 pages (:207-302);
* Prefill: raw K/V for PrefillNoCache, int8 pages on a cache hit (:304-368).

The quantise + scatter runs in one kernel (``qkv_int8_quant_store``) instead of
the reference's elementwise ops followed by the host's ``reshape_and_cache``.
"""

from __future__ import annotations

from typing import Any

import numpy as np
import torch


def _state_name(attn_metadata: Any) -> str:
    state = getattr(attn_metadata, "attn_state", None)
    if state is None:
        return "UNKNOWN"
    return getattr(state, "name", None) or str(state)


def _host_list(x) -> list[int]:
    if isinstance(x, torch.Tensor):
        return [int(v) for v in x.tolist()]
    return [int(v) for v in x]


class AscendInt8AttentionBackendMixin:
    """Runtime-calibrated INT8 KV cache on the B200 kernels."""

    key_cache: torch.Tensor | None = None
    value_cache: torch.Tensor | None = None

    def forward(self, layer: Any, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                kv_cache: Any, attn_metadata: Any, output: torch.Tensor | None = None,
                output_scale: torch.Tensor | None = None,
                output_block_scale: torch.Tensor | None = None) -> torch.Tensor:
        assert output is not None, "Output tensor must be provided."
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError(
                "fused output quantization is not yet supported for AscendInt8AttentionBackendImpl"
            )
        if attn_metadata is None:
            return output.fill_(0)
        if self.key_cache is None and kv_cache is not None and (
            (isinstance(kv_cache, torch.Tensor) and kv_cache.dim() > 0 and kv_cache.shape[0] == 2)
            or (isinstance(kv_cache, list | tuple) and len(kv_cache) >= 2)
        ):
            self.key_cache, self.value_cache = kv_cache[0], kv_cache[1]

        state = _state_name(attn_metadata)
        float_key = float_value = None
        if key is not None and value is not None:
            if state != "DecodeOnly":
                float_key, float_value = key, value
            self._prepare_int8_scales(layer, key, value)
            n = int(attn_metadata.num_actual_tokens)
            self._quantize_and_store_int8(key, value, layer, attn_metadata.slot_mapping, n)

        if getattr(attn_metadata, "model_runner_type", None) == "pooling" and not attn_metadata.causal:
            return self._forward_int8_dense(query, float_key, float_value, attn_metadata, output, causal=False)

        if not getattr(layer, "_int8_scales_ready", False):
            raise RuntimeError(
                "INT8 KV cache scales are not calibrated: the first forward of a layer must carry key/value"
            )
        if state == "DecodeOnly":
            return self._forward_int8_decode(query, attn_metadata, output, layer)
        if state == "ChunkedPrefill":
            return self._forward_int8_chunked_prefill(query, float_key, float_value, attn_metadata, output, layer)
        return self._forward_int8_prefill(query, float_key, float_value, attn_metadata, output, layer)

    # -- quantisation ---------------------------------------------------

    def _prepare_int8_scales(self, layer: Any, key: torch.Tensor, value: torch.Tensor) -> None:
        """Once per layer, from the first K/V passed in (attention_backend.py:130-150)."""
        if getattr(layer, "_int8_scales_ready", False):
            return
        from ...ops.int8 import int8_calc_scales

        k_inv, v_inv, k_aq, v_aq = int8_calc_scales(key, value)
        H, D = k_inv.shape
        layer._int8_k_inv_scale = k_inv.view(1, H, D)
        layer._int8_v_inv_scale = v_inv.view(1, H, D)
        layer._int8_k_offset = torch.zeros_like(layer._int8_k_inv_scale)
        layer._int8_v_offset = torch.zeros_like(layer._int8_v_inv_scale)
        layer._int8_k_aq_scale = k_aq.view(1, H, 1, D)
        layer._int8_v_aq_scale = v_aq.view(1, H, 1, D)
        layer._int8_k_aq_offset = layer._int8_k_offset.view(1, H, 1, D)
        layer._int8_v_aq_offset = layer._int8_v_offset.view(1, H, 1, D)
        layer._int8_scales_ready = True

    def _quantize_and_store_int8(self, key, value, layer, slot_mapping, num_actual_tokens: int) -> None:
        """Quantise the first ``num_actual_tokens`` K/V and write them at their
        slots (``_quantize_kv_to_runtime_int8`` + reshape_and_cache)."""
        from ...ops.int8 import int8_quant_store

        if self.key_cache is None or self.value_cache is None:
            raise RuntimeError("INT8 KV cache tensors are not bound.")
        n = num_actual_tokens
        H, D = layer._int8_k_inv_scale.shape[-2:]
        int8_quant_store(
            key[:n], value[:n], slot_mapping[:n],
            layer._int8_k_inv_scale.view(H, D), layer._int8_v_inv_scale.view(H, D),
            self.key_cache, self.value_cache,
        )

    # -- attention --------------------------------------------------------

    def _aq(self, layer):
        H, D = layer._int8_k_inv_scale.shape[-2:]
        return layer._int8_k_aq_scale.reshape(H, D), layer._int8_v_aq_scale.reshape(H, D)

    def _int8_device_i32(self, arr) -> torch.Tensor:
        t = torch.from_numpy(np.ascontiguousarray(arr, dtype=np.int32))
        return t.to(self.key_cache.device, non_blocking=True)

    def _int8_table(self, block_table, rows: int) -> torch.Tensor:
        dev = self.key_cache.device
        if isinstance(block_table, torch.Tensor):
            bt = block_table[:rows]
            if bt.device != dev:
                bt = bt.to(dev, non_blocking=True)
            return bt.to(torch.int32).contiguous()
        return self._int8_device_i32(np.asarray(block_table)[:rows])

    def _forward_int8_decode(self, query, attn_metadata, output, layer):
        """One query token per request over the int8 pages."""
        seq_lens = _host_list(attn_metadata.seq_lens_list)
        return self._int8_paged(query, attn_metadata.block_tables, seq_lens, output, layer)

    def _int8_paged(self, query, block_table, seq_lens, output, layer, rows_req=None):
        """Decode rows: query row i of ``query`` over ``seq_lens[i]`` keys of
        request ``rows_req[i]`` (row i itself when ``rows_req`` is None)."""
        from ...ops.int8 import int8_paged_decode

        B = len(seq_lens)
        if B == 0:
            return output
        k_aq, v_aq = self._aq(layer)
        bt = self._int8_table(block_table, (max(rows_req) + 1) if rows_req else B)
        if rows_req is not None:
            sel = torch.tensor(rows_req, dtype=torch.long).to(bt.device, non_blocking=True)
            bt = bt.index_select(0, sel).contiguous()
        int8_paged_decode(
            query[:B], self.key_cache, self.value_cache, k_aq, v_aq, bt, self._int8_device_i32(seq_lens),
            self.scale, output[:B], max(max(seq_lens), 1),
        )
        return output

    def _int8_history_rows(self, query, block_table, seq_lens, qlen, output, layer, causal=True):
        """Rows over the int8 pages (the dequantise-then-attend path of
        ``_dequant_int8_paged_kv_to_dense`` + FIA sparse_mode 3,
        attention_backend.py:282-302, :346-368). Requests with several query
        tokens gather their K/V densely and run the tensor-core prompt
        attention aligned to the end of their keys; single-token rows run the
        paged decode kernel with their causal length."""
        from ..history_rows import RowView, dense_prefill_geometry_ok, plan_history_rows

        B = len(qlen)
        plan = plan_history_rows(qlen, seq_lens[:B], causal,
                                 dense_prefill_geometry_ok(self.head_size, self.num_heads, self.num_kv_heads))
        if plan.num_tokens == 0:
            return output
        if plan.dense:
            self._int8_dense_history(query, block_table, plan, causal, output, layer)
        if not plan.rows_req:
            return output
        rows = RowView(query, output, plan.rows_q)
        self._int8_paged(rows.query, block_table, plan.rows_len, rows.output, layer, rows_req=plan.rows_req)
        rows.commit()
        return output

    def _int8_dense_history(self, query, block_table, plan, causal, output, layer):
        """Dense chunks of ``plan``: one gather of their int8 K/V and one
        prompt-attention launch over all of them."""
        from ...ops.int8 import int8_dequant_gather
        from ...ops.prefill import dense_prefill
        from ..history_rows import RowView

        reqs = plan.dense
        k_aq, v_aq = self._aq(layer)
        bt = self._int8_table(block_table, max(reqs) + 1)
        sel = torch.tensor(reqs, dtype=torch.long).to(bt.device, non_blocking=True)
        kv_lens = [plan.seq_lens[b] for b in reqs]
        dk, dv = int8_dequant_gather(self.key_cache, self.value_cache, k_aq, v_aq,
                                     bt.index_select(0, sel).contiguous(), kv_lens)
        rows = RowView(query, output, [plan.starts[b] + i for b in reqs for i in range(plan.q_lens[b])])
        dense_prefill(rows.query.contiguous(), dk, dv, [plan.q_lens[b] for b in reqs], kv_lens, self.scale,
                      rows.output, causal=causal)
        rows.commit()

    def _forward_int8_dense(self, query, key, value, attn_metadata, output, causal=True):
        from ...ops.prefill import dense_prefill

        qlen = _host_list(attn_metadata.actual_seq_lengths_q)
        n = int(qlen[-1])
        lens = [qlen[0]] + [qlen[i] - qlen[i - 1] for i in range(1, len(qlen))]
        dense_prefill(query[:n].contiguous(), key[:n].contiguous(), value[:n].contiguous(), lens, lens,
                      self.scale, output[:n], causal=causal)
        return output

    def _forward_int8_chunked_prefill(self, query, float_key, float_value, attn_metadata, output, layer):
        from ...ops.prefill import dense_prefill

        nd_tok = attn_metadata.num_decode_tokens
        nd = attn_metadata.num_decodes
        qlen = _host_list(attn_metadata.actual_seq_lengths_q)
        seq_lens = _host_list(attn_metadata.seq_lens_list)
        num_tokens = int(qlen[-1])
        if nd_tok > 0:
            self._int8_paged(query, attn_metadata.block_tables[:nd], seq_lens[:nd], output, layer)
        if attn_metadata.num_prefills <= 0:
            return output
        pre_q = [qlen[i] - nd_tok for i in range(nd, len(qlen))]
        lens = [pre_q[0]] + [pre_q[i] - pre_q[i - 1] for i in range(1, len(pre_q))]
        all_new = all(seq_lens[nd + i] <= lens[i] for i in range(len(lens)))
        if all_new and float_key is not None and float_value is not None:
            dense_prefill(query[nd_tok:num_tokens].contiguous(), float_key[nd_tok:num_tokens].contiguous(),
                          float_value[nd_tok:num_tokens].contiguous(), lens, lens, self.scale,
                          output[nd_tok:num_tokens], causal=True)
            return output
        sub = output[nd_tok:num_tokens]
        self._int8_history_rows(query[nd_tok:num_tokens], attn_metadata.block_tables[nd:], seq_lens[nd:],
                                pre_q, sub, layer)
        return output

    def _forward_int8_prefill(self, query, float_key, float_value, attn_metadata, output, layer):
        qlen = _host_list(attn_metadata.actual_seq_lengths_q)
        seq_lens = _host_list(attn_metadata.seq_lens_list)
        if _state_name(attn_metadata) == "PrefillNoCache" and float_key is not None:
            return self._forward_int8_dense(query, float_key, float_value, attn_metadata, output, causal=True)
        return self._int8_history_rows(query, attn_metadata.block_tables, seq_lens, qlen, output, layer)


__all__ = ["AscendInt8AttentionBackendMixin"]
