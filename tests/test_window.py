"""Host-planned residual windows vs the oracle's sequential state machine.

The mixin batches a forward's window updates into one plan (one gather, one
pack launch per side, one ring scatter); the reference walks tokens one by one.
Random operation sequences — bulk prefill, decode steps, in-place overwrites,
roll-backs, finished requests — must leave the same windows (slots and data)
and the same int4 history. Runs on CPU: the pack launches are recorded and
replayed through the oracle's packers."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import qkv_oracle as O
from qkv_b200.methods.kivi_int4.attention_backend import AscendKiviInt4AttentionBackendMixin
from qkv_b200.methods.kivi_int4.window import WindowPlanner


class _Stub:
    num_kv_heads = 2
    head_size = 32
    num_heads = 2
    num_queries_per_kv = 1
    scale = 0.125


def make_impl(group=8, residual=16, block=16, rows=4, nb=40):
    class Impl(AscendKiviInt4AttentionBackendMixin, _Stub):
        kivi_residual_dtype = torch.float32

    impl = Impl()
    impl._init_kivi_state(None)
    impl.enable_kivi = True
    impl.kivi_group_size = group
    impl.kivi_residual_length = residual
    impl.kivi_max_num_seqs = rows
    H, D = impl.num_kv_heads, impl.head_size
    impl.k_quant_cache = torch.zeros(nb, H, D, block // 8, dtype=torch.int32)
    impl.k_scale_cache = torch.ones(nb, H, D, block // group)
    impl.k_mn_cache = torch.zeros(nb, H, D, block // group)
    impl.v_quant_cache = torch.zeros(nb, block, H, D // 8, dtype=torch.int32)
    impl.v_scale_cache = torch.ones(nb, block, H, D // group)
    impl.v_mn_cache = torch.zeros(nb, block, H, D // group)
    impl.launches = []
    impl._launch_kivi_key_pack = lambda k, s: impl.launches.append((True, k.clone(), s.clone()))
    impl._launch_kivi_value_pack = lambda v, s: impl.launches.append((False, v.clone(), s.clone()))
    impl._launch_kivi_window_apply = _cpu_window_apply(impl)
    return impl


def _cpu_window_apply(impl):
    """The device apply of a plan restated with torch on CPU tensors (the
    GPU path is qkv_kivi_window_gather / qkv_kivi_window_scatter): every
    source is read before any ring lane is written, then packs, then the
    ring scatter."""

    def apply(exports, new_tokens):
        (kfs, kfl, kwl, kws), (vfs, vfl, vwl, vws) = exports
        rings = (impl.kivi_residual_key_cache, impl.kivi_residual_value_cache)
        taken = []
        for ring, new, fs, ws in ((rings[0], new_tokens[0], kfs, kws), (rings[1], new_tokens[1], vfs, vws)):
            flat = ring.view(-1, *ring.shape[2:])

            def take(src):
                rows = [flat[s].clone() if s >= 0 else new[-1 - s].clone() for s in src.tolist()]
                return torch.stack(rows) if rows else flat[:0].clone()

            taken.append((take(fs), take(ws)))
        if kfs.size:
            impl._write_kivi_key_quant_cache(taken[0][0], torch.from_numpy(kfl), _host_slots=kfl.tolist())
        if vfs.size:
            impl._write_kivi_value_quant_cache(taken[1][0], torch.from_numpy(vfl))
        for ring, wl, (_, data) in ((rings[0], kwl, taken[0]), (rings[1], vwl, taken[1])):
            if wl.size:
                ring.view(-1, *ring.shape[2:])[torch.from_numpy(wl)] = data

    return apply


def views_of(impl):
    return [t.numpy().copy() for t in impl._kivi_views()]


def apply_launches(impl, views, group):
    for is_key, data, slots in impl.launches:
        keep = slots.numpy() >= 0
        if is_key:
            O.kivi_pack_key(data.numpy()[keep], slots.numpy()[keep], *views[:3], group)
        else:
            O.kivi_pack_value(data.numpy(), slots.numpy(), *views[3:], group)
    impl.launches.clear()


def compare(impl, orc, views_impl, views_orc, reqs):
    for a, b in zip(views_impl, views_orc):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    for r in reqs:
        for is_key in (True, False):
            s1, t1 = impl._collect_kivi_residual_window(r, is_key=is_key)
            s2, t2 = orc.window(r, is_key)
            assert s1 == s2, (r, is_key)
            if s1:
                assert np.array_equal(t1.numpy(), np.stack(t2))


@pytest.mark.parametrize("seed", range(6))
def test_random_sequences_match_sequential_state_machine(seed):
    rng = np.random.default_rng(seed)
    group, residual, block, rows = 8, 16, 16, 4
    impl = make_impl(group, residual, block, rows)
    orc = O.ResidualOracle(capacity=residual, rows=rows, group_size=group, block_size=block)
    H, D = 2, 32
    vi, vo = views_of(impl), views_of(impl)
    reqs = ["r0", "r1", "r2"]
    tables = np.stack([rng.permutation(40)[:10] for _ in reqs])
    lens = {r: 0 for r in reqs}

    def slot(b, p):
        return int(tables[b, p // block]) * block + p % block

    # bulk prefill of ragged prompts (some exactly residual-sized)
    for b, r in enumerate(reqs):
        n = int(rng.choice([5, residual, 2 * residual + 3, 40]))
        k = rng.standard_normal((n, H, D)).astype(np.float32)
        v = rng.standard_normal((n, H, D)).astype(np.float32)
        sl = [slot(b, p) for p in range(n)]
        impl._write_kivi_prefill_cache(torch.from_numpy(k), torch.from_numpy(v), torch.tensor(sl), [r], [n])
        orc.write_prefill(r, k, v, sl)
        lens[r] = n
    apply_launches(impl, vi, group)
    orc.apply_flushes(vo)
    compare(impl, orc, vi, vo, reqs)

    for step in range(60):
        live = [b for b, r in enumerate(reqs) if r in lens]
        if not live:
            break
        # occasionally roll a request back, or rewrite its last token in place
        if rng.random() < 0.1:
            b = int(rng.choice(live))
            lens[reqs[b]] = max(1, lens[reqs[b]] - int(rng.integers(1, 5)))
        rewrite = rng.random() < 0.1
        B = len(live)
        k = rng.standard_normal((B, H, D)).astype(np.float32)
        v = rng.standard_normal((B, H, D)).astype(np.float32)
        sl = []
        for b in live:
            r = reqs[b]
            if not rewrite:
                lens[r] += 1
            sl.append(slot(b, lens[r] - 1))
        names = [reqs[b] for b in live]
        try:
            impl._write_kivi_cache(torch.from_numpy(k), torch.from_numpy(v), torch.tensor(sl), names,
                                   list(range(1, B + 1)))
        except RuntimeError as exc:
            # a roll-back can leave a key window that is no longer a run of
            # aligned groups: the reference fails closed on the same flush
            assert "aligned token groups" in str(exc)
            with pytest.raises(RuntimeError, match="aligned token groups"):
                orc.write_decode(names, k, v, sl)
            return
        orc.write_decode(names, k, v, sl)
        seq = [lens[r] for r in names]
        impl._sync_kivi_residual_windows(torch.from_numpy(tables[live]), seq, names)
        orc.sync(names, tables[live], seq)
        if step == 30:  # a request finishes
            impl._release_finished_kivi_residual_rows({"r1"})
            orc.release("r1")
            del lens["r1"]
        apply_launches(impl, vi, group)
        orc.apply_flushes(vo)
        compare(impl, orc, vi, vo, [r for r in reqs if r in lens])


def test_rows_lifecycle_and_exhaustion():
    impl = make_impl(rows=2)
    impl._ensure_kivi_residual_buffers()
    assert impl._get_kivi_residual_row("a", create=False) is None
    assert impl._get_kivi_residual_row("a", create=True) == 0
    impl._release_kivi_residual_row("a")
    assert impl.kivi_residual_free_rows == [1, 0]
    impl._get_kivi_residual_row("x", create=True)
    impl._get_kivi_residual_row("y", create=True)
    with pytest.raises(RuntimeError, match="exhausted"):
        impl._get_kivi_residual_row("z", create=True)


def test_key_window_flushes_whole_and_values_one_at_a_time():
    impl = make_impl(group=8, residual=16, block=16)
    key = torch.randn(16, 2, 32)
    impl._store_kivi_residual_entries(key, torch.arange(16), req_key="r", is_key=True)
    assert impl.launches == []
    impl._store_kivi_residual_entries(torch.randn(1, 2, 32), torch.tensor([32]), req_key="r", is_key=True)
    assert len(impl.launches) == 1 and impl.launches[0][2].tolist() == list(range(16))
    assert impl._collect_kivi_residual_window("r", is_key=True)[0] == [32]
    impl.launches.clear()
    val = torch.randn(17, 2, 32)
    impl._store_kivi_residual_entries(val, torch.arange(17), req_key="v", is_key=False)
    assert len(impl.launches) == 1 and impl.launches[0][2].tolist() == [0]
    assert impl._collect_kivi_residual_window("v", is_key=False)[0] == list(range(1, 17))


def test_bulk_prefill_flushes_full_window_but_incremental_keeps_it():
    tokens = 16
    key, value = torch.randn(tokens, 2, 32), torch.randn(tokens, 2, 32)
    bulk = make_impl()
    bulk._write_kivi_prefill_cache(key, value, torch.arange(tokens), ["b"], [tokens])
    assert [l[0] for l in bulk.launches] == [True, False]
    assert bulk._get_kivi_residual_row("b", create=False) is None
    inc = make_impl()
    for s in range(tokens):
        inc._write_kivi_cache(key[s:s + 1], value[s:s + 1], torch.tensor([s]), ["i"], [1])
    assert inc.launches == []
    row = inc._get_kivi_residual_row("i", create=False)
    assert inc.kivi_residual_key_len[row] == tokens and inc.kivi_residual_value_len[row] == tokens


def test_misaligned_key_flush_fails_before_any_launch():
    impl = make_impl()
    with pytest.raises(RuntimeError, match="aligned token groups"):
        impl._write_kivi_key_quant_cache(torch.randn(8, 2, 32), torch.arange(1, 9))
    with pytest.raises(RuntimeError, match="whole token groups"):
        impl._write_kivi_key_quant_cache(torch.randn(7, 2, 32), torch.arange(7))
    assert impl.launches == []


def test_forward_guards():
    impl = make_impl()
    out = torch.zeros(1, 2, 32)
    assert impl.forward(None, out, out, out, None, None, out) is out
    with pytest.raises(NotImplementedError, match="fused output quantization"):
        impl.forward(None, out, out, out, None, object(), out, output_scale=out)
    with pytest.raises(RuntimeError, match="6-tuple"):
        impl._bind_kivi_cache((impl.k_quant_cache,))
    impl.enable_kivi = False
    with pytest.raises(RuntimeError, match="kivi_int4 cache dtype"):
        impl.forward(None, out, out, out, None, object(), out)


def _plans_equal(a, b):
    return all(np.array_equal(x, y) for x, y in zip(a.export(), b.export()))


@pytest.mark.parametrize("seed", range(6))
def test_batched_decode_store_matches_per_row_store(seed):
    """store_one_each (one token per row, vectorised) leaves the same window
    state and plan as store() called row by row: appends, in-place hits,
    value evictions at capacity and whole-window key flushes."""
    rng = np.random.default_rng(seed)
    rows, cap, g, blk = 6, 8, 8, 16
    a, b = WindowPlanner(rows, cap, g), WindowPlanner(rows, cap, g)
    nxt = [int(r) * 4 * blk for r in range(rows)]  # each row owns 4 blocks, aligned start
    for _ in range(40):
        pa, pb = a.begin(), b.begin()
        rs = rng.permutation(rows)[: rng.integers(1, rows + 1)]
        slots = []
        for r in rs:
            if rng.random() < 0.2 and a.key.length[r] > 0:  # rewrite a held slot
                held = a.key.slots[r][a.key.slots[r] >= 0]
                slots.append(int(rng.choice(held)))
            else:
                slots.append(nxt[r])
                nxt[r] += 1
        tok = list(range(len(rs)))
        for is_key, i in ((True, 0), (False, 1)):
            for r, sl, t in zip(rs, slots, tok):
                a.store(pa[i], int(r), [sl], [t], is_key=is_key)
            b.store_one_each(pb[i], rs, slots, tok, is_key=is_key)
            assert _plans_equal(pa[i], pb[i])
        for side in ("key", "value"):
            sa, sb = getattr(a, side), getattr(b, side)
            assert np.array_equal(sa.slots, sb.slots)
            assert np.array_equal(sa.start, sb.start) and np.array_equal(sa.length, sb.length)


@pytest.mark.parametrize("seed", range(4))
def test_batched_liveness_matches_per_row(seed):
    rng = np.random.default_rng(100 + seed)
    rows, cap, g, blk = 5, 8, 8, 4
    pl = WindowPlanner(rows, cap, g)
    table = rng.permutation(40).reshape(5, 8).astype(np.int64)
    table[rng.random(table.shape) < 0.1] = -1
    lens = rng.integers(0, 8 * blk + 1, rows)
    for r in range(rows):
        for side in (pl.key, pl.value):
            n = int(rng.integers(0, cap + 1))
            st = int(rng.integers(0, cap))
            pos = np.arange(max(int(lens[r]) - n, 0), int(lens[r]))
            ids = table[r, pos // blk] * blk + pos % blk
            if rng.random() < 0.3 and ids.size:
                ids[rng.integers(0, ids.size)] += 1  # a stale entry
            side.slots[r].fill(-1)
            for i, v in enumerate(ids):
                side.slots[r, (st + i) % cap] = v
            side.start[r], side.length[r] = st, ids.size
    want = [_expected_live_py(pl, r, int(lens[r]), table[r], blk) for r in range(rows)]
    got = pl.expected_live_rows(np.arange(rows), lens, table, blk)
    assert got.tolist() == want


def _expected_live_py(pl, row, seq_len, table_row, blk):
    """Python restatement of the liveness check: window entry i of a window of
    n slots holds position seq_len - n + i."""
    for side in (pl.key, pl.value):
        lanes = side.lanes(row)
        n = len(lanes)
        if n == 0:
            continue
        if n > seq_len:
            return False
        pos = np.arange(seq_len - n, seq_len)
        if np.any(pos // blk >= table_row.size):
            return False
        blocks = table_row[pos // blk].astype(np.int64)
        if np.any(blocks < 0) or not np.array_equal(blocks * blk + pos % blk, side.slots[row, lanes]):
            return False
    return True
