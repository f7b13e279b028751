"""Pins the numpy oracle to the reference: golden vectors produced by running
the reference's own code (tests/golden/make_golden.py) must be reproduced
bit-exactly (codes, scales, mins, packed words) or, for attention, to fp32
rounding."""

from __future__ import annotations

import numpy as np
import pytest

import qkv_oracle as O
from conftest import bf16_to_f32


# ----------------------------------------------------------------- INT8


def test_int8_scales_bit_exact(golden):
    g = golden("int8")
    key, value = bf16_to_f32(g["key"]), bf16_to_f32(g["value"])
    k_inv, v_inv, k_aq, v_aq = O.int8_calc_scales(key, value)
    for got, want in ((k_inv, "k_inv"), (v_inv, "v_inv"), (k_aq, "k_aq"), (v_aq, "v_aq")):
        assert np.array_equal(O.bf16_bits(got), g[want]), want


def test_int8_codes_bit_exact(golden):
    g = golden("int8")
    n = int(g["n_actual"])
    key, value = bf16_to_f32(g["key"]), bf16_to_f32(g["value"])
    k_inv, v_inv = bf16_to_f32(g["k_inv"]), bf16_to_f32(g["v_inv"])
    assert np.array_equal(O.int8_quantize(key[:n], k_inv), g["k_codes"])
    assert np.array_equal(O.int8_quantize(value[:n], v_inv), g["v_codes"])


def test_int8_paged_store_and_dequant_bit_exact(golden):
    g = golden("int8")
    n = int(g["n_actual"])
    key, value = bf16_to_f32(g["key"]), bf16_to_f32(g["value"])
    k_inv, v_inv = bf16_to_f32(g["k_inv"]), bf16_to_f32(g["v_inv"])
    kc = np.zeros_like(g["key_cache"])
    vc = np.zeros_like(g["value_cache"])
    O.int8_quant_store(key[:n], value[:n], g["slots"], k_inv, v_inv, kc, vc)
    assert np.array_equal(kc, g["key_cache"]) and np.array_equal(vc, g["value_cache"])
    dk, dv = O.int8_dequant_gather(kc, vc, bf16_to_f32(g["k_aq"]), bf16_to_f32(g["v_aq"]),
                                   g["block_table"], g["seq_lens"])
    assert np.array_equal(O.bf16_bits(dk), g["dense_k"])
    assert np.array_equal(O.bf16_bits(dv), g["dense_v"])


def test_int8_roundtrip_within_resolution():
    """The reference's own known answer (tests/test_int8_dynamic.py:42-49)."""
    x = np.linspace(-1.0, 1.0, 32).astype(np.float32)
    q = O.int8_quantize(O.bf16_round(x), np.full_like(x, 127.0))
    assert q.dtype == np.int8
    assert np.max(np.abs(q.astype(np.float32) / 127.0 - x)) <= 1.0 / 127.0 + 1e-2


# ----------------------------------------------------------------- KIVI


def _geometries(g):
    return sorted({k.split("_")[0] for k in g if k.startswith("g") and k.endswith("_geometry")})


def test_kivi_pack_views_bit_exact_at_reference_geometries(golden):
    g = golden("kivi_pack")
    geoms = _geometries(g)
    assert len(geoms) == 5
    for p in geoms:
        head, kvh, group, block, residual, nb = g[p + "_geometry"].tolist()
        key, value = bf16_to_f32(g[p + "_key"]), bf16_to_f32(g[p + "_value"])
        slots = g[p + "_slots"]
        # initial state of the reference's _make_impl: scales 1, the rest 0
        views = [
            (np.ones_like if n.endswith("scale") else np.zeros_like)(g[f"{p}_{n}"])
            for n in ("k_quant", "k_scale", "k_mn", "v_quant", "v_scale", "v_mn")
        ]
        O.kivi_pack_key(key, slots, views[0], views[1], views[2], group)
        O.kivi_pack_value(value, slots, views[3], views[4], views[5], group)
        for v, n in zip(views, ("k_quant", "k_scale", "k_mn", "v_quant", "v_scale", "v_mn")):
            want = g[f"{p}_{n}"]
            assert v.dtype == want.dtype and np.array_equal(v.view(np.uint32), want.view(np.uint32)), (p, n)


def test_kivi_gather_matches_reference(golden):
    g = golden("kivi_pack")
    checked = 0
    for p in _geometries(g):
        if p + "_gather_k_f32" not in g:
            continue
        head, kvh, group, block, residual, nb = g[p + "_geometry"].tolist()
        views = [g[f"{p}_{n}"] for n in ("k_quant", "k_scale", "k_mn", "v_quant", "v_scale", "v_mn")]
        L = g[p + "_gather_k_f32"].shape[0]
        k32, v32 = O.kivi_dequant_gather(*views, g[p + "_block_table"], [L], group, target_bf16=False)
        assert np.array_equal(k32, g[p + "_gather_k_f32"]) and np.array_equal(v32, g[p + "_gather_v_f32"])
        k16, v16 = O.kivi_dequant_gather(*views, g[p + "_block_table"], [L], group, target_bf16=True)
        assert np.array_equal(O.bf16_bits(k16), g[p + "_gather_k_bf16"])
        assert np.array_equal(O.bf16_bits(v16), g[p + "_gather_v_bf16"])
        checked += 1
    assert checked >= 2


def test_kivi_pack_kernel_contract_known_answers():
    """Known answers of the reference's contract test
    (tests/test_kivi_int4.py:1140-1171): scale floor 1e-6, half-up ties, clip."""
    mn = np.zeros(1, np.float32)
    assert O.group_scale(mn, np.full(1, 3e-7, np.float32))[0] == pytest.approx(1e-6, rel=1e-6)
    assert O.group_scale(mn, np.full(1, 1e-9, np.float32))[0] == pytest.approx(1e-6, rel=1e-6)
    assert O.quantize_group(np.full(3, 2.5, np.float32), 0.0, np.float32(1.0)).tolist() == [3, 3, 3]
    assert O.quantize_group(np.full(1, 99.0, np.float32), 0.0, np.float32(1.0)).tolist() == [15]


def test_pack_unpack_roundtrip():
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 16, size=(3, 2, 4, 8))
    assert np.array_equal(O.unpack_int4(O.pack_int4(codes)), codes)


def test_fake_quant_matches_pack_then_gather():
    """fake_quant (the reference's CPU semantics) equals pack -> gather."""
    rng = np.random.default_rng(1)
    head, kvh, group, block = 32, 2, 8, 16
    key = O.bf16_round(rng.standard_normal((block, kvh, head)).astype(np.float32))
    val = O.bf16_round(rng.standard_normal((block, kvh, head)).astype(np.float32))
    views = [
        np.zeros((1, kvh, head, block // 8), np.int32), np.zeros((1, kvh, head, block // group), np.float32),
        np.zeros((1, kvh, head, block // group), np.float32), np.zeros((1, block, kvh, head // 8), np.int32),
        np.zeros((1, block, kvh, head // group), np.float32), np.zeros((1, block, kvh, head // group), np.float32),
    ]
    slots = np.arange(block)
    O.kivi_pack_key(key, slots, *views[:3], group)
    O.kivi_pack_value(val, slots, *views[3:], group)
    k, v = O.kivi_dequant_gather(*views, np.zeros((1, 1), np.int64), [block], group, target_bf16=False)
    assert np.array_equal(k, O.fake_quant_key(key, group))
    assert np.array_equal(v, O.fake_quant_value(val, group))


# ------------------------------------------------------ residual pipeline


def replay_pipeline(g):
    """Replays the golden KIVI pipeline with the oracle's state machine and
    attention; returns (views, oracle, per-step outputs)."""
    head, kvh, group, block, residual, nb, num_heads = g["geometry"].tolist()
    bt = g["block_table"]
    views = [
        np.zeros((nb, kvh, head, block // 8), np.int32), np.ones((nb, kvh, head, block // group), np.float32),
        np.zeros((nb, kvh, head, block // group), np.float32), np.zeros((nb, block, kvh, head // 8), np.int32),
        np.ones((nb, block, kvh, head // group), np.float32), np.zeros((nb, block, kvh, head // group), np.float32),
    ]
    orc = O.ResidualOracle(capacity=residual, rows=4, group_size=group, block_size=block)
    reqs = ["a", "b", "c"]
    pk, pv = bf16_to_f32(g["prefill_k"]), bf16_to_f32(g["prefill_v"])
    off = 0
    for b, n in enumerate(g["prompt_lens"].tolist()):
        slots = [int(bt[b, p // block]) * block + p % block for p in range(n)]
        orc.write_prefill(reqs[b], pk[off:off + n], pv[off:off + n], slots)
        off += n
    orc.apply_flushes(views)
    outs = []
    sq, sk, sv = bf16_to_f32(g["step_q"]), bf16_to_f32(g["step_k"]), bf16_to_f32(g["step_v"])
    for s in range(g["step_meta"].shape[0]):
        meta = g["step_meta"][s]
        live = [int(m[0]) for m in meta if m[0] >= 0]
        B = len(live)
        if any(int(m[3]) for m in meta if m[0] >= 0):
            orc.release("c")
        lens = [int(meta[i, 1]) for i in range(B)]
        slots = [int(meta[i, 2]) for i in range(B)]
        names = [reqs[i] for i in live]
        orc.write_decode(names, sk[s, :B], sv[s, :B], slots)
        orc.apply_flushes(views)
        orc.sync(names, bt[live], lens)
        dk, dv = O.kivi_dequant_gather(*views, bt[live], lens, group, target_bf16=False)
        kw = [np.asarray(orc.window(r, True)[1]) if orc.window(r, True)[1] else None for r in names]
        vw = [np.asarray(orc.window(r, False)[1]) if orc.window(r, False)[1] else None for r in names]
        dk, dv = O.overwrite_residual_tail(dk, dv, lens, kw, vw)
        outs.append(O.dense_attention(sq[s, :B], dk, dv, [1] * B, lens, head ** -0.5, causal=True))
    return views, orc, outs


def test_kivi_pipeline_oracle_matches_reference(golden):
    g = golden("kivi_pipeline")
    views, orc, outs = replay_pipeline(g)
    for v, n in zip(views, ("k_quant", "k_scale", "k_mn", "v_quant", "v_scale", "v_mn")):
        assert np.array_equal(v.view(np.uint32), g["final_" + n].view(np.uint32)), n
    for r in ("a", "b", "c"):
        for is_key, tag in ((True, "k"), (False, "v")):
            slots, data = orc.window(r, is_key)
            assert slots == g[f"final_win_{tag}_slots_{r}"].tolist(), (r, tag)
            if slots:
                assert np.array_equal(np.stack(data), g[f"final_win_{tag}_{r}"])
    for s, out in enumerate(outs):
        B = out.shape[0]
        np.testing.assert_allclose(out, g["step_out"][s, :B], atol=2e-5, rtol=0)


def test_ordered_slots_and_alignment_known_cases():
    """Cases of the reference's tests (tests/test_kivi_int4.py:127-190)."""
    assert O.is_aligned_key_window(list(range(16, 24)) + list(range(32, 40)), 8, 16)
    assert not O.is_aligned_key_window([], 8, 16)
    assert not O.is_aligned_key_window(list(range(1, 9)), 8, 16)
    assert not O.is_aligned_key_window(list(range(12, 20)), 8, 16)
    table = np.array([[3, -1, 5]])
    assert O.ordered_slots(table, [70], 32) == [list(range(96, 128)) + list(range(160, 166))]
    assert O.ordered_slots(np.array([[3, 4]]), [0], 32) == [[]]
