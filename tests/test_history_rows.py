"""Host-side row planning of the paths over cached keys (no GPU)."""

from __future__ import annotations

from qkv_b200.methods.history_rows import dense_prefill_geometry_ok, plan_history_rows


def test_multi_token_requests_become_dense_chunks():
    # two decode rows, then chunks of 64 and 33 tokens
    plan = plan_history_rows([1, 2, 66, 99], [701, 301, 1064, 162], causal=True, dense_ok=True)
    assert plan.starts == [0, 1, 2, 66] and plan.q_lens == [1, 1, 64, 33]
    assert plan.dense == [2, 3]
    assert plan.rows_req == [0, 1] and plan.rows_len == [701, 301] and plan.rows_q == [0, 1]
    assert plan.num_tokens == 99


def test_without_dense_every_token_is_a_row_with_its_causal_length():
    plan = plan_history_rows([3, 4], [10, 5], causal=True, dense_ok=False)
    assert plan.dense == []
    assert plan.rows_req == [0, 0, 0, 1]
    assert plan.rows_len == [8, 9, 10, 5]  # query i of 3 over 10 keys sees 10 - 3 + i + 1
    assert plan.rows_q == [0, 1, 2, 3]
    flat = plan_history_rows([3], [10], causal=False, dense_ok=False)
    assert flat.rows_len == [10, 10, 10]


def test_empty_requests_and_zero_lengths():
    plan = plan_history_rows([0, 2, 2], [0, 7, 0], causal=True, dense_ok=True)
    assert plan.dense == [1] and plan.rows_req == []
    none = plan_history_rows([], [], causal=True, dense_ok=True)
    assert none.num_tokens == 0


def test_dense_geometry():
    assert dense_prefill_geometry_ok(128, 32, 8) and dense_prefill_geometry_ok(128, 8, 8)
    assert dense_prefill_geometry_ok(128, 64, 8)
    assert not dense_prefill_geometry_ok(128, 40, 8)  # 5 query heads per KV head
    assert not dense_prefill_geometry_ok(64, 32, 8)
    assert not dense_prefill_geometry_ok(128, 128, 8)  # 16 per KV head
