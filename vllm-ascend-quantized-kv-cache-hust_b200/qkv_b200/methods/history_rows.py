"""Host-side row planning shared by the INT8 and KIVI paths over cached keys.

The reference attends every multi-token request over cached keys through one
dequantise-then-attend call aligned to the end of its keys (FIA sparse_mode 3;
methods/int8_dynamic/attention_backend.py:246-368,
methods/kivi_int4/attention_backend.py:1157-1191). Here a request with several
query tokens becomes a dense chunk (gather + tensor-core prompt attention) when
the geometry allows it; every other query token becomes a decode row with its
causal length.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


def dense_prefill_geometry_ok(head_size: int, num_heads: int, num_kv_heads: int) -> bool:
    """Geometry of the tcgen05 prompt attention: head 128 and 1, 2, 4 or 8
    query heads per KV head."""
    return head_size == 128 and num_heads % num_kv_heads == 0 and num_heads // num_kv_heads in (1, 2, 4, 8)


@dataclass
class HistoryPlan:
    starts: list[int]  # first query row of each request
    q_lens: list[int]
    seq_lens: list[int]
    dense: list[int] = field(default_factory=list)  # requests run as dense chunks
    rows_req: list[int] = field(default_factory=list)  # decode rows: request,
    rows_len: list[int] = field(default_factory=list)  # causal length,
    rows_q: list[int] = field(default_factory=list)  # query row

    @property
    def num_tokens(self) -> int:
        return self.starts[-1] + self.q_lens[-1] if self.starts else 0


def plan_history_rows(qlen_cumulative, seq_lens, causal: bool, dense_ok: bool) -> HistoryPlan:
    """``qlen_cumulative``: cumulative query ends per request
    (``actual_seq_lengths_q``); ``seq_lens``: keys per request including the
    new tokens. Query token i of a request with q_len tokens over L keys sees
    keys [0, L - q_len + i] when causal, all L otherwise."""
    starts, q_lens = [], []
    prev = 0
    for q_end in qlen_cumulative:
        starts.append(prev)
        q_lens.append(int(q_end) - prev)
        prev = int(q_end)
    lens = [int(s) for s in seq_lens]
    plan = HistoryPlan(starts, q_lens, lens)
    if dense_ok:
        plan.dense = [b for b in range(len(lens)) if q_lens[b] > 1 and lens[b] > 0]
    dense_set = set(plan.dense)
    for b, L in enumerate(lens):
        if b in dense_set:
            continue
        ql = q_lens[b]
        for i in range(ql):
            plan.rows_req.append(b)
            plan.rows_len.append(max(0, min(L, L - ql + i + 1)) if causal else L)
            plan.rows_q.append(starts[b] + i)
    return plan


class RowView:
    """Query / output rows of a subset: slices of the caller's tensors when the
    rows are consecutive, gathered copies otherwise (``commit`` scatters the
    output rows back)."""

    def __init__(self, query: torch.Tensor, output: torch.Tensor, rows: list[int]) -> None:
        self._output = output
        self._index = None
        n = len(rows)
        if rows == list(range(rows[0], rows[0] + n)):
            self.query = query[rows[0]:rows[0] + n]
            self.output = output[rows[0]:rows[0] + n]
        else:
            self._index = torch.tensor(rows, dtype=torch.long).to(query.device, non_blocking=True)
            self.query = query.index_select(0, self._index).contiguous()
            self.output = torch.empty((n,) + tuple(output.shape[1:]), dtype=output.dtype, device=output.device)

    def commit(self) -> None:
        if self._index is not None:
            self._output.index_copy_(0, self._index, self.output)


__all__ = ["HistoryPlan", "RowView", "dense_prefill_geometry_ok", "plan_history_rows"]
