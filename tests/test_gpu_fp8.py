"""FP8 per-token-head device path vs the oracle (pinned to the reference's
semantics): store bit-exact, gather bit-exact, decode attention within the
attention tolerance, on the TMA geometry (head 128, page 128) and the generic
one."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import qkv_oracle as O
from conftest import bf16_to_f32

pytestmark = pytest.mark.gpu
ATOL = 1e-2


def dev():
    return torch.device("cuda", 0)


def close(got, want, atol=ATOL):
    assert np.isfinite(got).all()
    err = np.abs(got - want) - (atol + np.abs(want) * 2.0 ** -8)
    assert err.max() <= 0, float(np.abs(got - want).max())


def assert_no_device_error():
    from qkv_b200.ops import _lib

    assert _lib.device_error(torch.cuda.current_stream().cuda_stream) == 0


def views(nb, blk, H, D):
    f = lambda *s, dt: torch.zeros(*s, dtype=dt, device=dev())
    return (f(nb, blk, H, D, dt=torch.uint8), f(nb, blk, H, 1, dt=torch.float32),
            f(nb, blk, H, D, dt=torch.uint8), f(nb, blk, H, 1, dt=torch.float32))


def test_store_matches_reference_golden(golden):
    from qkv_b200.ops import fp8_store

    g = golden("fp8")
    T, H, D, blk, nb = g["geometry"].tolist()
    v = views(nb, blk, H, D)
    k = torch.from_numpy(bf16_to_f32(g["key"])).to(dev()).bfloat16()
    val = torch.from_numpy(bf16_to_f32(g["value"])).to(dev()).bfloat16()
    fp8_store(k, val, torch.from_numpy(g["slots"]).to(dev()), *v)
    slots = g["slots"]
    assert np.array_equal(v[0].view(nb * blk, H, D)[torch.from_numpy(slots)].cpu().numpy(), g["k_codes"])
    assert np.array_equal(v[1].view(nb * blk, H, 1)[torch.from_numpy(slots)].cpu().numpy().view(np.uint32),
                          g["k_scale"].view(np.uint32))
    assert np.array_equal(v[2].view(nb * blk, H, D)[torch.from_numpy(slots)].cpu().numpy(), g["v_codes"])
    assert_no_device_error()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("slot_dtype", [torch.int32, torch.int64])
def test_store_bit_exact_random(dtype, slot_dtype):
    from qkv_b200.ops import fp8_store

    rng = np.random.default_rng(3)
    T, H, D, blk, nb = 3000, 8, 128, 128, 40
    mag = np.exp(rng.uniform(-9, 5, (T, H, 1)))
    k = torch.from_numpy((rng.standard_normal((T, H, D)) * mag).astype(np.float32)).to(dtype)
    vv = torch.from_numpy((rng.standard_normal((T, H, D)) * mag).astype(np.float32)).to(dtype)
    k[7] = 0
    slots = rng.permutation(nb * blk)[:T].astype(np.int64)
    slots[::97] = -1
    v = views(nb, blk, H, D)
    fp8_store(k.to(dev()), vv.to(dev()), torch.from_numpy(slots).to(dev(), slot_dtype), *v)
    want = [np.zeros(tuple(t.shape), dtype=np.uint8 if t.dtype == torch.uint8 else np.float32) for t in v]
    O.fp8_store(k.float().numpy(), vv.float().numpy(), slots, *want)
    for got, w in zip(v, want):
        assert np.array_equal(got.cpu().numpy().view(np.uint8), w.view(np.uint8))
    assert_no_device_error()


def _paged_case(rng, lens, H, D, blk):
    B = len(lens)
    maxp = max((L + blk - 1) // blk for L in lens)
    nb = B * maxp + 2
    bt = rng.permutation(nb)[:B * maxp].reshape(B, maxp).astype(np.int32)
    v = [np.zeros((nb, blk, H, D), np.uint8), np.zeros((nb, blk, H, 1), np.float32),
         np.zeros((nb, blk, H, D), np.uint8), np.zeros((nb, blk, H, 1), np.float32)]
    for b, L in enumerate(lens):
        pos = np.arange(L)
        slots = bt[b, pos // blk].astype(np.int64) * blk + pos % blk
        # per-(token, head) magnitudes: keys e^U(-1, 1) (logits up to about
        # +-10: the fp16 query fragment keeps them within the tolerance),
        # values e^U(-2, 2)
        kmag = np.exp(rng.uniform(-1, 1, (L, H, 1))).astype(np.float32)
        vmag = np.exp(rng.uniform(-2, 2, (L, H, 1))).astype(np.float32)
        K = O.bf16_round((rng.standard_normal((L, H, D)) * kmag).astype(np.float32))
        V = O.bf16_round((rng.standard_normal((L, H, D)) * vmag).astype(np.float32))
        O.fp8_store(K, V, slots, *v)
    return v, bt


@pytest.mark.parametrize("lens,Hq,H,D,blk", [
    ([1, 127, 128, 3000, 8192], 32, 8, 128, 128),  # TMA kernel, GQA 4
    ([5000, 77], 64, 8, 128, 128),                 # GQA 8
    ([16384], 8, 8, 128, 128),                     # GQA 1, long
    ([40, 300, 1], 4, 2, 64, 16),                  # generic kernel
])
def test_decode_vs_oracle(lens, Hq, H, D, blk):
    from qkv_b200.ops import fp8_paged_decode

    rng = np.random.default_rng(sum(lens) + D)
    v, bt = _paged_case(rng, lens, H, D, blk)
    B = len(lens)
    q = O.bf16_round(rng.standard_normal((B, Hq, D)).astype(np.float32))
    tv = [torch.from_numpy(x).to(dev()) for x in v]
    out = torch.full((B, Hq, D), float("nan"), dtype=torch.bfloat16, device=dev())
    fp8_paged_decode(torch.from_numpy(q).to(dev()).bfloat16(), *tv, torch.from_numpy(bt).to(dev()),
                     torch.tensor(lens, dtype=torch.int32, device=dev()), D ** -0.5, out, max(lens))
    dk, dv = O.fp8_dequant_gather(*v, bt, lens, target_bf16=False)
    want = O.dense_attention(q, dk, dv, [1] * B, lens, D ** -0.5, causal=True)
    close(out.float().cpu().numpy(), want)
    assert_no_device_error()


def test_gather_bit_exact():
    from qkv_b200.ops import fp8_dequant_gather

    rng = np.random.default_rng(12)
    lens, H, D, blk = [1, 129, 4000], 8, 128, 128
    v, bt = _paged_case(rng, lens, H, D, blk)
    tv = [torch.from_numpy(x).to(dev()) for x in v]
    dk, dv = fp8_dequant_gather(*tv, torch.from_numpy(bt).to(dev()), lens)
    wk, wv = O.fp8_dequant_gather(*v, bt, lens, target_bf16=True)
    assert np.array_equal(dk.float().cpu().numpy().view(np.uint32), wk.view(np.uint32))
    assert np.array_equal(dv.float().cpu().numpy().view(np.uint32), wv.view(np.uint32))
    assert_no_device_error()


def test_fp8_mixin_prompts_chunks_and_decode_match_oracle():
    """The FP8 mixin over the host's two byte buffers: a PrefillNoCache batch
    (attention over the raw K/V), a ChunkedPrefill batch with two decode rows
    and two chunks over cached tokens, a PrefillCacheHit batch and a
    DecodeOnly batch over the pages; every row matches the oracle's
    dequantise-then-attend over the pages after the write."""
    from types import SimpleNamespace

    from qkv_b200.methods.fp8_per_token_head.attention_backend import AscendFp8PerTokenHeadAttentionBackendMixin
    from qkv_b200.methods.fp8_per_token_head.byte_cache import Fp8PerTokenHeadLayout

    H, Hq, D, blk, nb = 8, 32, 128, 128, 64

    class Impl(AscendFp8PerTokenHeadAttentionBackendMixin):
        pass

    impl = Impl()
    impl.num_heads, impl.num_kv_heads, impl.head_size, impl.num_queries_per_kv = Hq, H, D, Hq // H
    impl.scale = D ** -0.5
    lay = Fp8PerTokenHeadLayout(num_blocks=nb, block_size=blk, num_kv_heads=H, head_size=D)
    raw = torch.zeros(2, nb, blk, H, lay.bytes_per_token_head, dtype=torch.uint8, device=dev())
    bt = torch.arange(48, dtype=torch.int32).reshape(4, 12)
    rng = np.random.default_rng(81)
    bf = lambda *s: torch.from_numpy(O.bf16_round(rng.standard_normal(s).astype(np.float32))).to(dev()).bfloat16()

    def slots(b, lo, hi):
        return torch.tensor([int(bt[b, p // blk]) * blk + p % blk for p in range(lo, hi)], device=dev())

    before = [0, 0, 0, 0]

    def run(state, reqs, ql, **extra):
        lens = [before[b] + n for b, n in zip(reqs, ql)]
        T = sum(ql)
        q, k, v = bf(T, Hq, D), bf(T, H, D), bf(T, H, D)
        md = SimpleNamespace(
            attn_state=SimpleNamespace(name=state), actual_seq_lengths_q=np.cumsum(ql).tolist(),
            seq_lens_list=lens, slot_mapping=torch.cat([slots(b, before[b], L) for b, L in zip(reqs, lens)]),
            block_tables=bt[reqs].to(dev()), num_actual_tokens=T, causal=True, **extra,
        )
        out = torch.full((T, Hq, D), float("nan"), dtype=torch.bfloat16, device=dev())
        impl.forward(None, q, k, v, raw, md, out)
        for b, L in zip(reqs, lens):
            before[b] = L
        return q, k, v, out, lens

    prompts = [700, 300, 1000, 129]
    q, k, v, out, _ = run("PrefillNoCache", [0, 1, 2, 3], prompts)
    want = O.dense_attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                             prompts, prompts, D ** -0.5, causal=True)
    close(out.float().cpu().numpy(), want)
    views = [t.cpu().numpy() for t in (impl.k_data, impl.k_scale, impl.v_data, impl.v_scale)]
    for state, reqs, ql, extra in (
        ("ChunkedPrefill", [0, 1, 2, 3], [1, 1, 64, 33], dict(num_decode_tokens=2, num_decodes=2, num_prefills=2)),
        ("PrefillCacheHit", [2, 0], [50, 1], {}),
        ("DecodeOnly", [0, 1, 2, 3], [1, 1, 1, 1], {}),
    ):
        q, _, _, out, lens = run(state, reqs, ql, **extra)
        views = [t.cpu().numpy() for t in (impl.k_data, impl.k_scale, impl.v_data, impl.v_scale)]
        dk, dv = O.fp8_dequant_gather(*views, bt[reqs].numpy(), lens, target_bf16=True)
        want = O.dense_attention(q.float().cpu().numpy(), dk, dv, ql, lens, D ** -0.5, causal=True)
        close(out.float().cpu().numpy(), want)
    assert_no_device_error()
