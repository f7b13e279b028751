"""The KIVI mixin end to end on the GPU against the reference's own pipeline.

Replays tests/golden/kivi_pipeline.npz — recorded by running the reference's
``AscendKiviInt4AttentionBackendMixin.forward`` — through this package's
mixin on CUDA: bulk prefill writes, 40 decode steps with key-window flushes,
value evictions, a finished request and a roll-back. The int4 history must be
bit-identical, the windows identical, and every step's attention output within
1e-2 of the reference's."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import bf16_to_f32
from qkv_b200.methods.kivi_int4.attention_backend import AscendKiviInt4AttentionBackendMixin

pytestmark = pytest.mark.gpu
ATOL = 1e-2


def make_impl(g, device):
    head, kvh, group, block, residual, nb, num_heads = g["geometry"].tolist()

    class Host:
        pass

    class Impl(AscendKiviInt4AttentionBackendMixin, Host):
        pass

    impl = Impl()
    impl.num_heads, impl.num_kv_heads, impl.head_size = num_heads, kvh, head
    impl.num_queries_per_kv = num_heads // kvh
    impl.scale = head ** -0.5
    impl._init_kivi_state(
        "kivi_int4",
        SimpleNamespace(
            cache_config=SimpleNamespace(kivi_group_size=group, kivi_residual_length=residual),
            scheduler_config=SimpleNamespace(max_num_seqs=4),
        ),
    )
    f = lambda *s, dt=torch.float32, v=0.0: torch.full(s, v, dtype=dt, device=device)
    six = (
        f(nb, kvh, head, block // 8, dt=torch.int32), f(nb, kvh, head, block // group, v=1.0),
        f(nb, kvh, head, block // group), f(nb, block, kvh, head // 8, dt=torch.int32),
        f(nb, block, kvh, head // group, v=1.0), f(nb, block, kvh, head // group),
    )
    return impl, six


@pytest.mark.parametrize("state", ["PrefillCacheHit", "DecodeOnly"])
def test_mixin_forward_reproduces_reference_pipeline(golden, state):
    g = golden("kivi_pipeline")
    dev = torch.device("cuda", 0)
    head, kvh, group, block, residual, nb, num_heads = g["geometry"].tolist()
    impl, six = make_impl(g, dev)
    impl._bind_kivi_cache(six)
    bt = torch.from_numpy(g["block_table"])
    reqs = ["a", "b", "c"]
    pk = torch.from_numpy(bf16_to_f32(g["prefill_k"])).to(dev).to(torch.bfloat16)
    pv = torch.from_numpy(bf16_to_f32(g["prefill_v"])).to(dev).to(torch.bfloat16)
    off = 0
    for b, n in enumerate(g["prompt_lens"].tolist()):
        slots = torch.tensor([int(bt[b, p // block]) * block + p % block for p in range(n)], device=dev)
        impl._write_kivi_prefill_cache(pk[off:off + n], pv[off:off + n], slots, [reqs[b]], [n])
        off += n
    sq, sk, sv = (bf16_to_f32(g[n]) for n in ("step_q", "step_k", "step_v"))
    for s in range(g["step_meta"].shape[0]):
        meta = g["step_meta"][s]
        live = [int(m[0]) for m in meta if m[0] >= 0]
        B = len(live)
        finished = {"c"} if any(int(m[3]) for m in meta[:B]) else None
        md = SimpleNamespace(
            attn_state=SimpleNamespace(name=state),
            actual_seq_lengths_q=list(range(1, B + 1)),
            seq_lens_list=[int(meta[i, 1]) for i in range(B)],
            slot_mapping=torch.tensor([int(meta[i, 2]) for i in range(B)], device=dev),
            block_tables=bt[live].to(dev),
            req_ids=[reqs[i] for i in live],
            num_actual_tokens=B,
            causal=True,
            finished_req_ids=finished,
        )
        q = torch.from_numpy(sq[s, :B]).to(dev).to(torch.bfloat16)
        k = torch.from_numpy(sk[s, :B]).to(dev).to(torch.bfloat16)
        v = torch.from_numpy(sv[s, :B]).to(dev).to(torch.bfloat16)
        out = torch.zeros(B, num_heads, head, dtype=torch.bfloat16, device=dev)
        impl.forward(None, q, k, v, six, md, out)
        err = (out.float().cpu().numpy() - g["step_out"][s, :B]).__abs__().max()
        assert err <= ATOL, (s, err)
    for t, n in zip(six, ("k_quant", "k_scale", "k_mn", "v_quant", "v_scale", "v_mn")):
        assert np.array_equal(t.cpu().numpy().view(np.uint32), g["final_" + n].view(np.uint32)), n
    for r in reqs:
        for is_key, tag in ((True, "k"), (False, "v")):
            slots, data = impl._collect_kivi_residual_window(r, is_key=is_key)
            assert slots == g[f"final_win_{tag}_slots_{r}"].tolist(), (r, tag)
            if slots:
                assert np.array_equal(data.float().cpu().numpy(), g[f"final_win_{tag}_{r}"])


def test_mixin_on_host_byte_buffers_matches_six_views(golden):
    """The host's two byte buffers give the same result as a 6-tuple."""
    from qkv_b200.methods.kivi_int4.byte_cache import KiviByteCacheLayout

    dev = torch.device("cuda", 0)
    torch.manual_seed(5)
    H, D, g_, blk, r, nb = 2, 32, 8, 16, 16, 4
    lay = KiviByteCacheLayout(num_blocks=nb, block_size=blk, num_kv_heads=H, head_size=D, group_size=g_)
    kbuf = torch.zeros(nb, blk, H, lay.bytes_per_token_head, dtype=torch.uint8, device=dev)
    vbuf = torch.zeros_like(kbuf)
    fake = {"geometry": np.array([D, H, g_, blk, r, nb, H])}
    impl, six = make_impl(fake, dev)
    impl2, _ = make_impl(fake, dev)
    tokens = r + 1
    q = torch.randn(tokens, H, D, device=dev).to(torch.bfloat16)
    k = torch.randn(tokens, H, D, device=dev).to(torch.bfloat16)
    v = torch.randn(tokens, H, D, device=dev).to(torch.bfloat16)
    md = SimpleNamespace(
        attn_state=SimpleNamespace(name="PrefillCacheHit"), actual_seq_lengths_q=[tokens],
        seq_lens_list=[tokens], slot_mapping=torch.arange(tokens, device=dev),
        block_tables=torch.tensor([[0, 1]], device=dev), req_ids=["r"], num_actual_tokens=tokens, causal=True,
        finished_req_ids=None,
    )
    o1 = torch.zeros(tokens, H, D, dtype=torch.bfloat16, device=dev)
    o2 = torch.zeros_like(o1)
    for t in six:  # byte buffers start at zero: make the 6-tuple start there too
        t.zero_()
    impl.forward(None, q, k, v, six, md, o1)
    impl2.forward(None, q, k, v, (kbuf, vbuf), md, o2)
    assert torch.equal(o1, o2)
    assert kbuf.any() and vbuf.any()


def test_mixin_chunk_over_history_matches_oracle():
    """Prefill chunks on cached tokens next to a single-token row (head 128,
    4 query heads per KV head): chunks run gather + tensor-core attention, the
    single row the paged decode kernel; every output row matches the oracle's
    dequantise-to-bf16-then-attend over the cache state after the write."""
    import qkv_oracle as O

    dev = torch.device("cuda", 0)
    head, kvh, group, block, residual, nb, num_heads = 128, 8, 128, 128, 128, 64, 32
    impl, six = make_impl({"geometry": np.array([head, kvh, group, block, residual, nb, num_heads])}, dev)
    impl._bind_kivi_cache(six)
    rng = np.random.default_rng(3)
    reqs, prompt, ql = ["a", "b", "c"], [1000, 300, 777], [64, 1, 40]
    bt = torch.arange(48, dtype=torch.int32).reshape(3, 16)
    bf = lambda *s: torch.from_numpy(O.bf16_round(rng.standard_normal(s).astype(np.float32))).to(dev).bfloat16()

    def slots(b, lo, hi):
        return torch.tensor([int(bt[b, p // block]) * block + p % block for p in range(lo, hi)], device=dev)

    for b, n in enumerate(prompt):
        impl._write_kivi_prefill_cache(bf(n, kvh, head), bf(n, kvh, head), slots(b, 0, n), [reqs[b]], [n])
    lens = [p + n for p, n in zip(prompt, ql)]
    T = sum(ql)
    q, k, v = bf(T, num_heads, head), bf(T, kvh, head), bf(T, kvh, head)
    md = SimpleNamespace(
        attn_state=SimpleNamespace(name="PrefillCacheHit"), actual_seq_lengths_q=np.cumsum(ql).tolist(),
        seq_lens_list=lens, slot_mapping=torch.cat([slots(b, prompt[b], lens[b]) for b in range(3)]),
        block_tables=bt.to(dev), req_ids=reqs, num_actual_tokens=T, causal=True, finished_req_ids=None,
    )
    out = torch.full((T, num_heads, head), float("nan"), dtype=torch.bfloat16, device=dev)
    impl.forward(None, q, k, v, six, md, out)
    views = [t.cpu().numpy() for t in six]
    wins = {}
    for tag, is_key in (("k", True), ("v", False)):
        wins[tag] = []
        for r in reqs:
            _, data = impl._collect_kivi_residual_window(r, is_key=is_key)
            wins[tag].append(None if data is None or len(data) == 0 else data.float().cpu().numpy())
    dk, dv = O.kivi_dequant_gather(*views, bt.numpy(), lens, group, target_bf16=True)
    dk, dv = O.overwrite_residual_tail(dk, dv, lens, wins["k"], wins["v"])
    want = O.dense_attention(q.float().cpu().numpy(), dk, dv, ql, lens, head ** -0.5, causal=True)
    err = np.abs(out.float().cpu().numpy() - want).max()
    assert err <= ATOL, err


def test_int8_mixin_prompts_then_chunks_over_history_match_oracle():
    """INT8 mixin, three batches: PrefillNoCache calibrates the scales and
    fills the pages (attention over the raw K/V); ChunkedPrefill with two
    decode rows and two chunks over cached tokens, and PrefillCacheHit, read
    the int8 pages (chunks through the int8 gather + tensor-core attention,
    single rows through the paged decode kernel). Every row matches the
    oracle's dequantise-to-bf16-then-attend over the pages after the write."""
    import qkv_oracle as O
    from qkv_b200.methods.int8_dynamic.attention_backend import AscendInt8AttentionBackendMixin

    dev = torch.device("cuda", 0)
    H, Hq, D, blk, nb = 8, 32, 128, 128, 64

    class Impl(AscendInt8AttentionBackendMixin):
        pass

    impl = Impl()
    impl.num_heads, impl.num_kv_heads, impl.head_size, impl.num_queries_per_kv = Hq, H, D, Hq // H
    impl.scale = D ** -0.5
    layer = SimpleNamespace()
    cache = torch.zeros(2, nb, blk, H, D, dtype=torch.int8, device=dev)
    bt = torch.arange(48, dtype=torch.int32).reshape(4, 12)
    rng = np.random.default_rng(8)
    bf = lambda *s: torch.from_numpy(O.bf16_round(rng.standard_normal(s).astype(np.float32))).to(dev).bfloat16()

    def slots(b, lo, hi):
        return torch.tensor([int(bt[b, p // blk]) * blk + p % blk for p in range(lo, hi)], device=dev)

    def run(state, reqs, ql, before, **extra):
        lens = [before[b] + n for b, n in zip(reqs, ql)]
        T = sum(ql)
        q, k, v = bf(T, Hq, D), bf(T, H, D), bf(T, H, D)
        md = SimpleNamespace(
            attn_state=SimpleNamespace(name=state), actual_seq_lengths_q=np.cumsum(ql).tolist(),
            seq_lens_list=lens, slot_mapping=torch.cat([slots(b, before[b], L) for b, L in zip(reqs, lens)]),
            block_tables=bt[reqs].to(dev), num_actual_tokens=T, causal=True, **extra,
        )
        out = torch.full((T, Hq, D), float("nan"), dtype=torch.bfloat16, device=dev)
        impl.forward(layer, q, k, v, cache, md, out)
        for b, L in zip(reqs, lens):
            before[b] = L
        return q, k, v, out, lens

    before = [0, 0, 0, 0]
    prompts = [700, 300, 1000, 129]
    q, k, v, out, _ = run("PrefillNoCache", [0, 1, 2, 3], prompts, before)
    want = O.dense_attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                             prompts, prompts, D ** -0.5, causal=True)
    assert np.abs(out.float().cpu().numpy() - want).max() <= ATOL

    k_aq = layer._int8_k_aq_scale.reshape(H, D).float().cpu().numpy()
    v_aq = layer._int8_v_aq_scale.reshape(H, D).float().cpu().numpy()
    for state, reqs, ql, extra in (
        ("ChunkedPrefill", [0, 1, 2, 3], [1, 1, 64, 33],
         dict(num_decode_tokens=2, num_decodes=2, num_prefills=2)),
        ("PrefillCacheHit", [2, 0], [50, 1], {}),
    ):
        q, _, _, out, lens = run(state, reqs, ql, before, **extra)
        dk, dv = O.int8_dequant_gather(cache[0].cpu().numpy(), cache[1].cpu().numpy(), k_aq, v_aq,
                                       bt[reqs].numpy(), lens, target_bf16=True)
        want = O.dense_attention(q.float().cpu().numpy(), dk, dv, ql, lens, D ** -0.5, causal=True)
        err = np.abs(out.float().cpu().numpy() - want).max()
        assert err <= ATOL, (state, err)


def test_int8_dequant_gather_bit_exact():
    """Dense K/V from the int8 pages equal the oracle's gather (code * aq,
    one bf16 rounding) bit for bit, block tables shuffled, ragged lengths."""
    import qkv_oracle as O
    from qkv_b200.ops import int8_dequant_gather

    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(9)
    H, D, blk, lens = 8, 128, 128, [1, 127, 128, 129, 3000]
    maxp = max((L + blk - 1) // blk for L in lens)
    nb = len(lens) * maxp + 3
    kc = rng.integers(-128, 128, (nb, blk, H, D), dtype=np.int8)
    vc = rng.integers(-128, 128, (nb, blk, H, D), dtype=np.int8)
    aq = O.bf16_round(rng.uniform(0.001, 0.2, (2, H, D)).astype(np.float32))
    bt = rng.permutation(nb)[:len(lens) * maxp].reshape(len(lens), maxp).astype(np.int32)
    t = lambda x: torch.from_numpy(x).to(dev)
    dk, dv = int8_dequant_gather(t(kc), t(vc), t(aq[0]).bfloat16(), t(aq[1]).bfloat16(), t(bt), lens)
    wk, wv = O.int8_dequant_gather(kc, vc, aq[0], aq[1], bt, lens, target_bf16=True)
    assert np.array_equal(dk.float().cpu().numpy().view(np.uint32), wk.astype(np.float32).view(np.uint32))
    assert np.array_equal(dv.float().cpu().numpy().view(np.uint32), wv.astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("table_on", ["device", "host"])
def test_native_decode_step_matches_general_path(table_on):
    """qkv_kivi_decode_step (planning, sync and launches in one native call)
    against the general Python-planned path on the same decode sequence:
    bulk prompt writes, 140 decode steps crossing key-window flushes, value
    evictions, a roll-back of 3 tokens and a finished request. Outputs, int4
    pages and windows must be identical bit for bit. The block table comes
    on the device, or on the host (pinned; the step then stages it with its
    indices)."""
    dev = torch.device("cuda", 0)
    head, kvh, group, block, residual, nb, num_heads = 128, 8, 64, 128, 128, 40, 32
    geo = {"geometry": np.array([head, kvh, group, block, residual, nb, num_heads])}
    native, six_a = make_impl(geo, dev)
    general, six_b = make_impl(geo, dev)
    general._kivi_native_decode = lambda *a, **k: False
    calls = []
    orig = native._kivi_native_decode
    native._kivi_native_decode = lambda *a, **k: calls.append(orig(*a, **k)) or calls[-1]
    rng = np.random.default_rng(21)
    reqs, prompt = ["a", "b", "c"], [250, 127, 300]
    bt = torch.arange(36, dtype=torch.int32).reshape(3, 12)
    bf = lambda *s: torch.from_numpy(rng.standard_normal(s).astype(np.float32)).to(dev).bfloat16()

    def slot(b, p):
        return int(bt[b, p // block]) * block + p % block

    for impl, six in ((native, six_a), (general, six_b)):
        impl._bind_kivi_cache(six)
    for b, n in enumerate(prompt):
        k, v = bf(n, kvh, head), bf(n, kvh, head)
        sl = torch.tensor([slot(b, p) for p in range(n)], device=dev)
        for impl in (native, general):
            impl._write_kivi_prefill_cache(k, v, sl, [reqs[b]], [n])
    lens = list(prompt)
    live = [0, 1, 2]
    for step in range(140):
        if step == 70:
            lens[1] -= 3  # roll back request b by 3 tokens
        if step == 100:
            live = [0, 2]  # request b finishes
        for b in live:
            lens[b] += 1
        B = len(live)
        q, k, v = bf(B, num_heads, head), bf(B, kvh, head), bf(B, kvh, head)
        outs = []
        for impl, six in ((native, six_a), (general, six_b)):
            md = SimpleNamespace(
                attn_state=SimpleNamespace(name="DecodeOnly"), actual_seq_lengths_q=list(range(1, B + 1)),
                seq_lens_list=[lens[b] for b in live],
                slot_mapping=torch.tensor([slot(b, lens[b] - 1) for b in live], device=dev),
                block_tables=bt[live].to(dev) if table_on == "device" else bt[live].pin_memory(),
                req_ids=[reqs[b] for b in live], num_actual_tokens=B, causal=True,
                finished_req_ids={"b"} if step == 100 else None,
            )
            out = torch.zeros(B, num_heads, head, dtype=torch.bfloat16, device=dev)
            impl.forward(None, q, k, v, six, md, out)
            outs.append(out)
        assert torch.equal(outs[0], outs[1]), step
    assert calls and all(calls)
    for ta, tb in zip(six_a, six_b):
        assert torch.equal(ta, tb)
    for r in ("a", "c"):
        for is_key in (True, False):
            sa, da = native._collect_kivi_residual_window(r, is_key=is_key)
            sb, db = general._collect_kivi_residual_window(r, is_key=is_key)
            assert sa == sb and torch.equal(da, db), (r, is_key)
