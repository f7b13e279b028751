"""CPU oracle of the quantized-KV attention path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference plugin's own CPU arithmetic for
the hot path (paths relative to ``src/vllm_ascend_quantized_kv_cache/`` of the
reference project). It is the checker the CUDA kernels are compared against;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import it, and nothing in the product package does.

Pinning: every function here is checked against golden vectors produced by
running the reference itself (``tests/golden/make_golden.py`` imports the
reference's Python package and its CPU test packers; the fixtures live in
``tests/golden/*.npz``), see ``tests/test_oracle_golden.py``.

Numerics: all arithmetic is float32 with IEEE round-to-nearest, in the same
operation order as the torch CPU ops it restates; bf16 values are carried as
float32 numbers that are exactly representable in bf16 (``bf16_round``).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

F32 = np.float32


# ---------------------------------------------------------------------------
# bf16 emulation
# ---------------------------------------------------------------------------


def bf16_round(x) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32, like torch's ``.to(bf16)``."""
    x = np.ascontiguousarray(np.asarray(x, dtype=F32))
    b = x.view(np.uint32).astype(np.uint64)
    rounded = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(F32).reshape(x.shape)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, x, out)
    return out


def bf16_bits(x) -> np.ndarray:
    """uint16 bit patterns of bf16 values held in float32."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(F32)


# ---------------------------------------------------------------------------
# INT8 dynamic per-channel (methods/int8_dynamic/attention_backend.py:130-171,
# :370-404; semantics.py:49-83)
# ---------------------------------------------------------------------------


def int8_calc_scales(key: np.ndarray, value: np.ndarray):
    """Per-(head, channel) scales from the first K/V batch of a layer.

    Follows ``_prepare_int8_scales`` (attention_backend.py:138-147) evaluated on
    bf16 tensors: ``amax.clamp(min=1e-12)``, then ``127.0 / amax`` which torch
    computes as ``reciprocal(amax) * 127`` with a bf16 rounding after each op,
    then ``1.0 / inv`` for the BNSD antiquant scale.
    Inputs hold bf16 values ``[T, H, D]``; returns (k_inv, v_inv, k_aq, v_aq),
    each ``[H, D]`` float32 holding bf16 values.
    """

    def one(x):
        amax = np.abs(np.asarray(x, F32)).max(axis=0)
        amax = np.maximum(amax, bf16_round(F32(1e-12)))
        rec = bf16_round(F32(1.0) / amax)
        inv = bf16_round(rec * F32(127.0))
        aq = bf16_round(F32(1.0) / inv)
        return inv, aq

    k_inv, k_aq = one(key)
    v_inv, v_aq = one(value)
    return k_inv, v_inv, k_aq, v_aq


def int8_quantize(x: np.ndarray, inv: np.ndarray) -> np.ndarray:
    """``clamp(round(x * inv + 0), -128, 127).to(int8)`` on bf16 operands
    (attention_backend.py:161-170): the product is rounded to bf16, adding the
    zero offset is exact, ``torch.round`` is half-to-even like ``np.rint``."""
    prod = bf16_round(np.asarray(x, F32) * np.asarray(inv, F32))
    return np.clip(np.rint(prod), -128, 127).astype(np.int8)


def int8_quant_store(key, value, slots, k_inv, v_inv, key_cache, value_cache):
    """Quantise and scatter into ``[NB, blk, H, D]`` int8 pages by slot
    (the host's reshape_and_cache after ``_quantize_kv_to_runtime_int8``);
    negative slots are padding and skipped."""
    nb, blk = key_cache.shape[:2]
    kq = int8_quantize(key, k_inv)
    vq = int8_quantize(value, v_inv)
    for t, slot in enumerate(np.asarray(slots).tolist()):
        if slot < 0:
            continue
        key_cache[slot // blk, slot % blk] = kq[t]
        value_cache[slot // blk, slot % blk] = vq[t]


def int8_dequant_gather(key_cache, value_cache, k_aq, v_aq, block_table, seq_lens, target_bf16: bool = True):
    """``_dequant_int8_paged_kv_to_dense`` (attention_backend.py:370-404):
    gather live tokens by block table and dequantise ``code * aq``, rounded to
    bf16 as the reference's bf16 tensors are (``target_bf16=False`` keeps the
    exact fp32 products). Returns dense K, V ``[sum(seq_lens), H, D]``."""
    blk = key_cache.shape[1]
    ks, vs = [], []
    for b, L in enumerate(seq_lens):
        pos = np.arange(int(L))
        pages = np.asarray(block_table)[b, pos // blk]
        ks.append(key_cache[pages, pos % blk].astype(F32))
        vs.append(value_cache[pages, pos % blk].astype(F32))
    k = np.concatenate(ks) if ks else np.zeros((0,) + key_cache.shape[2:], F32)
    v = np.concatenate(vs) if vs else np.zeros((0,) + value_cache.shape[2:], F32)
    k, v = k * k_aq, v * v_aq
    return (bf16_round(k), bf16_round(v)) if target_bf16 else (k, v)


# ---------------------------------------------------------------------------
# FP8 per-token-head (methods/fp8_per_token_head/semantics.py:36-72,
# byte_cache.py:1-196)
# ---------------------------------------------------------------------------

E4M3_MAX = F32(448.0)
FP8_SCALE_FLOOR = F32(1e-6)


def e4m3_encode(x) -> np.ndarray:
    """float32 -> E4M3 (fn: 1 sign, 4 exponent bits with bias 7, 3 mantissa
    bits, subnormals, no infinities, 0x7F/0xFF NaN, max normal 448) bytes,
    round to nearest even — the conversion torch's ``.to(float8_e4m3fn)``
    performs. Inputs must lie in [-448, 448] (the semantics clamp first)."""
    x = np.asarray(x, F32)
    a = np.abs(x).astype(np.float64)
    if np.any(a > 448.0) or np.any(np.isnan(a)):
        raise ValueError("e4m3_encode expects finite inputs within [-448, 448]")
    sign = (np.signbit(x)).astype(np.uint8) << 7
    mant, exp = np.frexp(a)  # a = mant * 2^exp, mant in [0.5, 1)
    e = exp.astype(np.int64) - 1  # a = (2 mant) * 2^e, 2 mant in [1, 2)
    normal = (a > 0) & (e >= -6)
    # normal: 3 mantissa bits of (a / 2^e - 1); rounding may carry into the exponent
    frac = np.where(normal, (a / np.ldexp(1.0, np.clip(e, -6, 8)) - 1.0) * 8.0, 0.0)
    m = np.round(frac)  # half to even
    e_adj = np.where(m >= 8, e + 1, e)
    m = np.where(m >= 8, 0, m)
    norm_bits = ((e_adj + 7) << 3) | m.astype(np.int64)
    # subnormal: units of 2^-9
    sub = np.round(a / 2.0 ** -9).astype(np.int64)  # 8 -> 0b0001000 = 2^-6, the smallest normal
    bits = np.where(normal, norm_bits, sub)
    return (bits.astype(np.uint8) | sign).reshape(x.shape)


def e4m3_decode(b) -> np.ndarray:
    """E4M3 bytes -> float32 (exact)."""
    b = np.asarray(b, np.uint8).astype(np.int64)
    sign = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.ldexp(1.0, e - 7))
    val = np.where((e == 15) & (m == 7), np.nan, val)
    return (sign * val).astype(F32)


def fp8_quantize(x):
    """``Fp8PerTokenHeadSemantics.quantize`` (semantics.py:61-66): per
    (token, head) ``scale = max(amax / 448, 1e-6)``, ``e4m3(clamp(x / scale,
    -448, 448))``; x ``[T, H, D]`` -> (bytes ``[T, H, D]`` uint8, scale
    ``[T, H, 1]`` float32)."""
    x = np.asarray(x, F32)
    amax = np.abs(x).max(axis=-1, keepdims=True)
    scale = np.maximum(amax / E4M3_MAX, FP8_SCALE_FLOOR).astype(F32)
    q = np.clip(x / scale, -E4M3_MAX, E4M3_MAX).astype(F32)
    return e4m3_encode(q), scale


def fp8_dequantize(codes, scale):
    """``Fp8PerTokenHeadSemantics.dequantize`` (semantics.py:68-70)."""
    return (e4m3_decode(codes) * np.asarray(scale, F32)).astype(F32)


def fp8_store(key, value, slots, k_data, k_scale, v_data, v_scale):
    """Per-token-head store into the paged views (data ``[NB, blk, H, D]``
    uint8, scale ``[NB, blk, H, 1]`` float32); slots < 0 are skipped."""
    blk = k_data.shape[1]
    for x, data, sc in ((key, k_data, k_scale), (value, v_data, v_scale)):
        q, s = fp8_quantize(x)
        for t, slot in enumerate(np.asarray(slots).tolist()):
            if slot < 0:
                continue
            data[slot // blk, slot % blk] = q[t]
            sc[slot // blk, slot % blk] = s[t]


def fp8_dequant_gather(k_data, k_scale, v_data, v_scale, block_table, seq_lens, target_bf16: bool = True):
    """Dense K, V ``[sum L, H, D]`` of whole requests from the fp8 pages
    (``code * scale`` in fp32, then bf16 as the attention inputs are)."""
    blk = k_data.shape[1]
    ks, vs = [], []
    bt = np.asarray(block_table)
    for b, L in enumerate(seq_lens):
        pos = np.arange(int(L))
        pages, off = bt[b, pos // blk], pos % blk
        ks.append(fp8_dequantize(k_data[pages, off], k_scale[pages, off]))
        vs.append(fp8_dequantize(v_data[pages, off], v_scale[pages, off]))
    H, D = k_data.shape[2:]
    k = np.concatenate(ks) if ks else np.zeros((0, H, D), F32)
    v = np.concatenate(vs) if vs else np.zeros((0, H, D), F32)
    return (bf16_round(k), bf16_round(v)) if target_bf16 else (k, v)


# ---------------------------------------------------------------------------
# KIVI INT4 arithmetic (methods/kivi_int4/semantics.py:63-111;
# ops/triton/kivi_pack.py:61-226)
# ---------------------------------------------------------------------------


def group_scale(mn, mx):
    """``max((mx - mn) / 15, 1e-6)`` in fp32 (semantics.py:85-93)."""
    return np.maximum((np.asarray(mx, F32) - np.asarray(mn, F32)) / F32(15.0), F32(1e-6))


def quantize_group(x, mn, scale):
    """``clamp(floor((x - mn) / scale + 0.5), 0, 15)`` (semantics.py:95-111)."""
    q = np.floor((np.asarray(x, F32) - mn) / scale + F32(0.5))
    return np.clip(q, 0, 15).astype(np.int32)


def pack_int4(codes: np.ndarray) -> np.ndarray:
    """8 lanes (last dim) -> one int32 word, lane L at bits 4L (semantics.py:76-83)."""
    c = np.asarray(codes).astype(np.uint32) & 0xF
    word = np.zeros(c.shape[:-1], np.uint32)
    for lane in range(8):
        word |= c[..., lane] << np.uint32(4 * lane)
    return word.view(np.int32)


def unpack_int4(words: np.ndarray) -> np.ndarray:
    """int32 word -> 8 int4 lanes (new last dim) (semantics.py:63-74)."""
    w = np.asarray(words).view(np.uint32) if np.asarray(words).dtype == np.int32 else np.asarray(words, np.uint32)
    return np.stack([(w >> np.uint32(4 * lane)) & 0xF for lane in range(8)], axis=-1).astype(np.int32)


def kivi_pack_key(key, slots, k_quant, k_scale, k_mn, group_size):
    """Whole-group key pack (ops/triton/kivi_pack.py:134-226): per (token group,
    head, channel) min/max over the group's tokens, 8 consecutive tokens per
    word at ``k_quant[blk, h, d, (off + 8j)/8]``, scale/min at
    ``k_scale[blk, h, d, off/g]``. ``key`` is ``[n*g, H, D]`` float32."""
    key = np.asarray(key, F32)
    slots = np.asarray(slots).astype(np.int64)
    g = group_size
    blk = k_quant.shape[-1] * 8
    for gi in range(key.shape[0] // g):
        first = int(slots[gi * g])
        if first < 0:
            continue
        b, off = first // blk, first % blk
        grp = key[gi * g:(gi + 1) * g]  # [g, H, D]
        mn = grp.min(axis=0)
        mx = grp.max(axis=0)
        scale = group_scale(mn, mx)
        codes = quantize_group(grp, mn[None], scale[None])  # [g, H, D]
        words = pack_int4(codes.transpose(1, 2, 0).reshape(codes.shape[1], codes.shape[2], g // 8, 8))
        k_quant[b, :, :, off // 8: off // 8 + g // 8] = words
        k_scale[b, :, :, off // g] = scale
        k_mn[b, :, :, off // g] = mn


def kivi_pack_value(value, slots, v_quant, v_scale, v_mn, group_size):
    """Per-token value pack (ops/triton/kivi_pack.py:61-131): head_size split in
    groups of g, 8 dims per word at ``v_quant[blk, off, h, dim/8]``."""
    value = np.asarray(value, F32)
    slots = np.asarray(slots).astype(np.int64)
    g = group_size
    blk = v_quant.shape[1]
    T, H, D = value.shape
    grouped = value.reshape(T, H, D // g, g)
    mn = grouped.min(axis=-1)
    mx = grouped.max(axis=-1)
    scale = group_scale(mn, mx)
    codes = quantize_group(grouped, mn[..., None], scale[..., None]).reshape(T, H, D // 8, 8)
    words = pack_int4(codes)
    for t, slot in enumerate(slots.tolist()):
        if slot < 0:
            continue
        v_quant[slot // blk, slot % blk] = words[t]
        v_scale[slot // blk, slot % blk] = scale[t]
        v_mn[slot // blk, slot % blk] = mn[t]


def fake_quant_key(key, group_size):
    """``KiviInt4Semantics.fake_quant_key`` (semantics.py:113-135)."""
    key = np.asarray(key, F32)
    T = key.shape[0]
    if T == 0:
        return key
    pad = (group_size - T % group_size) % group_size
    work = np.concatenate([key, np.repeat(key[-1:], pad, axis=0)]) if pad else key
    grp = work.reshape(-1, group_size, *key.shape[1:])
    mn = grp.min(axis=1, keepdims=True)
    scale = group_scale(mn, grp.max(axis=1, keepdims=True))
    q = quantize_group(grp, mn, scale)
    deq = (q.astype(F32) * scale + mn).reshape(-1, *key.shape[1:])
    return deq[:T]


def fake_quant_value(value, group_size):
    """``KiviInt4Semantics.fake_quant_value`` (semantics.py:137-154)."""
    value = np.asarray(value, F32)
    D = value.shape[-1]
    grp = value.reshape(*value.shape[:-1], D // group_size, group_size)
    mn = grp.min(axis=-1, keepdims=True)
    scale = group_scale(mn, grp.max(axis=-1, keepdims=True))
    q = quantize_group(grp, mn, scale)
    return (q.astype(F32) * scale + mn).reshape(value.shape)


def kivi_dequant_gather(k_quant, k_scale, k_mn, v_quant, v_scale, v_mn, block_table, seq_lens, group_size,
                        target_bf16: bool = True):
    """``kivi_dequant_gather_cache`` (ops/kivi_gather.py:36-156): gather each
    request's pages, unpack, ``q * scale + mn`` in fp32 (two roundings), keep
    live tokens, cast to the target dtype. Returns dense K, V ``[sum L, H, D]``."""
    NB, H, D, wpb = k_quant.shape
    blk = wpb * 8
    g = group_size
    ks, vs = [], []
    bt = np.asarray(block_table)
    for b, L in enumerate(seq_lens):
        L = int(L)
        if L == 0:
            continue
        pos = np.arange(L)
        pages = bt[b, pos // blk]
        off = pos % blk
        # keys: [L, H, D]
        words = k_quant[pages, :, :, off // 8]  # [L, H, D]
        codes = (words.view(np.uint32) >> (4 * (off % 8)).astype(np.uint32)[:, None, None]) & 0xF
        sc = k_scale[pages, :, :, off // g]
        mn = k_mn[pages, :, :, off // g]
        ks.append(codes.astype(F32) * sc + mn)
        # values: [L, H, D]
        vw = v_quant[pages, off]  # [L, H, D/8]
        vcodes = unpack_int4(vw).reshape(L, H, D)
        vsc = np.repeat(v_scale[pages, off], g, axis=-1)
        vmn = np.repeat(v_mn[pages, off], g, axis=-1)
        vs.append(vcodes.astype(F32) * vsc + vmn)
    k = np.concatenate(ks) if ks else np.zeros((0, H, D), F32)
    v = np.concatenate(vs) if vs else np.zeros((0, H, D), F32)
    if target_bf16:
        k, v = bf16_round(k), bf16_round(v)
    return k, v


def overwrite_residual_tail(dense_k, dense_v, seq_lens, k_windows, v_windows):
    """Residual-tail overwrite of ``_gather_dequant_kivi_paged_cache``
    (methods/kivi_int4/attention_backend.py:889-935): the last len(window)
    positions of each request take the exact window values (FIFO order)."""
    dense_k = dense_k.copy()
    dense_v = dense_v.copy()
    start = 0
    for b, L in enumerate(seq_lens):
        L = int(L)
        for dense, win in ((dense_k, k_windows[b]), (dense_v, v_windows[b])):
            if win is not None and len(win) > 0 and L > 0:
                n = min(L, len(win))
                dense[start + L - n:start + L] = np.asarray(win, F32)[-n:]
        start += L
    return dense_k, dense_v


def dense_attention(q, k, v, q_lens, kv_lens, scale, causal=True):
    """fp32 restatement of ``_forward_kivi_dense_attention``
    (methods/kivi_int4/attention_backend.py:1341-1392) with the additive mask of
    ``build_causal_mask`` (semantics.py:285-299): query i of a request with
    q_len queries over kv_len keys sees key j iff j <= kv_len - q_len + i.
    q ``[sum q_lens, Hq, D]``, k/v ``[sum kv_lens, H, D]`` -> out like q."""
    q = np.asarray(q, F32)
    k = np.asarray(k, F32)
    v = np.asarray(v, F32)
    Hq, H = q.shape[1], k.shape[1]
    rep = Hq // H
    out = np.zeros_like(q)
    qs = ks = 0
    for ql, kl in zip(q_lens, kv_lens):
        ql, kl = int(ql), int(kl)
        if ql > 0 and kl > 0:
            qq = q[qs:qs + ql].transpose(1, 0, 2)  # [Hq, ql, D]
            kk = np.repeat(k[ks:ks + kl], rep, axis=1).transpose(1, 2, 0)  # [Hq, D, kl]
            vv = np.repeat(v[ks:ks + kl], rep, axis=1).transpose(1, 0, 2)  # [Hq, kl, D]
            s = np.matmul(qq, kk) * F32(scale)
            if causal:
                qpos = np.arange(kl - ql, kl)[:, None]
                kpos = np.arange(kl)[None, :]
                s = np.where(kpos > qpos, -np.inf, s)
            s = s - s.max(axis=-1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=-1, keepdims=True)
            out[qs:qs + ql] = np.matmul(p, vv).transpose(1, 0, 2)
        qs += ql
        ks += kl
    return out


def kivi_decode_reference(views, block_table, seq_lens, k_windows, v_windows, q, group_size, scale,
                          target_bf16: bool = True):
    """One decode query per request through the reference's KIVI read path:
    ``kivi_dequant_gather_cache`` (ops/kivi_gather.py:36-156) with the cast to
    the query dtype (bf16; ``target_bf16=False`` keeps the fp32 values), the
    residual-tail overwrite (methods/kivi_int4/attention_backend.py:889-935),
    then attention in fp32 (``dense_attention``)."""
    dk, dv = kivi_dequant_gather(*views, block_table, seq_lens, group_size, target_bf16=target_bf16)
    dk, dv = overwrite_residual_tail(dk, dv, seq_lens, k_windows, v_windows)
    return dense_attention(q, dk, dv, [1] * len(seq_lens), seq_lens, scale, causal=True)


def int8_decode_reference(key_cache, value_cache, k_aq, v_aq, block_table, seq_lens, q, scale,
                          target_bf16: bool = True):
    """One decode query per request through the reference's INT8 dense
    dequantisation (methods/int8_dynamic/attention_backend.py:370-404, bf16
    ``code * aq`` unless ``target_bf16=False``), then fp32 attention."""
    dk, dv = int8_dequant_gather(key_cache, value_cache, k_aq, v_aq, block_table, seq_lens,
                                 target_bf16=target_bf16)
    return dense_attention(q, dk, dv, [1] * len(seq_lens), seq_lens, scale, causal=True)


# Attention parity bound: max-abs 1e-2 wherever a bf16 output can resolve it.
# The outputs (the reference's and these kernels') are bf16; for |want| >= 2
# adjacent bf16 values are more than 1e-2 apart (2^-6 in [2, 4), 2^-5 in
# [4, 8), ...), so there the bound is one bf16 step of the reference value.
ATTN_ATOL = 1e-2


def bf16_spacing(x) -> np.ndarray:
    """Distance between adjacent bf16 values around |x|: 2^(e - 7) for |x| in
    [2^e, 2^(e + 1))."""
    a = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return np.exp2(e - 7)


def attention_error(got, want, atol: float = ATTN_ATOL) -> dict:
    """Errors of bf16 attention outputs ``got`` against reference values
    ``want``: the max-abs error overall and where bf16 resolves ``atol``
    (|want| < 2), how many outputs lie beyond that resolution, and whether
    every output is within max(atol, one bf16 step of want)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    d = np.abs(got - want)
    bound = np.maximum(atol, bf16_spacing(want))
    small = np.abs(want) < 2.0
    return {
        "max_abs": float(d.max()) if d.size else 0.0,
        "max_abs_where_bf16_resolves_1e-2": float(d[small].max()) if small.any() else 0.0,
        "outputs": int(d.size),
        "outputs_abs_ge_2": int((~small).sum()),
        "worst_excess_over_bound": float((d - bound).max()) if d.size else 0.0,
        "within_bound": bool(np.isfinite(got).all() and (d <= bound).all()),
    }


# ---------------------------------------------------------------------------
# Residual-window state machine (methods/kivi_int4/attention_backend.py:181-462,
# :562-674, :813-836; semantics.py:224-283) — pure Python, small cases
# ---------------------------------------------------------------------------


def ordered_slots(block_table, seq_lens, block_size):
    """``KiviInt4Semantics.ordered_slots`` (semantics.py:224-252)."""
    bt = np.asarray(block_table).astype(np.int64)
    out = []
    for b, L in enumerate(seq_lens):
        L = int(L)
        pos = np.arange(L)
        if L == 0:
            out.append([])
            continue
        s = bt[b, pos // block_size] * block_size + pos % block_size
        out.append([int(x) for x in s[s >= 0]])
    return out


def is_aligned_key_window(slots, group_size, block_size):
    """``KiviInt4Semantics.is_aligned_key_window`` (semantics.py:254-283)."""
    if not slots or len(slots) % group_size:
        return False
    for i in range(0, len(slots), group_size):
        grp = [int(s) for s in slots[i:i + group_size]]
        first = grp[0]
        if first % block_size % group_size:
            return False
        if grp[-1] // block_size != first // block_size:
            return False
        if grp != list(range(first, first + group_size)):
            return False
    return True


@dataclass
class _Row:
    slots: list  # lane -> slot or None
    data: list   # lane -> np.ndarray [H, D] or None
    start: int = 0
    length: int = 0


@dataclass
class ResidualOracle:
    """Per-request residual windows with the reference's asymmetric eviction:
    keys flush the whole window when a new slot arrives at a full window,
    values evict one oldest slot (attention_backend.py:411-462); bulk prefill
    flushes ``floor(n / r) * r`` tokens directly (:608-674).

    ``flushes`` records every pack launch as (is_key, slots, values)."""

    capacity: int
    rows: int
    group_size: int
    block_size: int
    key_rows: dict = field(default_factory=dict)
    val_rows: dict = field(default_factory=dict)
    req_to_row: dict = field(default_factory=dict)
    free_rows: list = field(default_factory=list)
    flushes: list = field(default_factory=list)

    def __post_init__(self):
        self.free_rows = list(range(self.rows - 1, -1, -1))

    def _row(self, req, create):
        r = self.req_to_row.get(req)
        if r is not None or not create:
            return r
        if not self.free_rows:
            raise RuntimeError("KIVI residual rows are exhausted.")
        r = self.free_rows.pop()
        self.req_to_row[req] = r
        self.key_rows[r] = _Row([None] * self.capacity, [None] * self.capacity)
        self.val_rows[r] = _Row([None] * self.capacity, [None] * self.capacity)
        return r

    def release(self, req):
        r = self.req_to_row.pop(req, None)
        if r is None:
            return
        self.key_rows.pop(r, None)
        self.val_rows.pop(r, None)
        self.free_rows.append(r)

    def _lanes(self, row: _Row):
        return [(row.start + i) % self.capacity for i in range(row.length)]

    def window(self, req, is_key):
        r = self.req_to_row.get(req)
        if r is None:
            return [], []
        row = (self.key_rows if is_key else self.val_rows)[r]
        lanes = self._lanes(row)
        return [row.slots[l] for l in lanes], [row.data[l] for l in lanes]

    def _flush(self, row: _Row, is_key, count):
        lanes = self._lanes(row)[:count]
        slots = [row.slots[l] for l in lanes]
        data = [row.data[l] for l in lanes]
        if is_key and not is_aligned_key_window(slots, self.group_size, self.block_size):
            raise RuntimeError("KIVI key flush requires contiguous aligned token groups.")
        self.flushes.append((is_key, slots, np.stack(data)))
        for l in lanes:
            row.slots[l] = None
            row.data[l] = None
        row.length -= count
        row.start = 0 if row.length == 0 else (row.start + count) % self.capacity

    def store(self, req, values, slots, is_key):
        if len(slots) == 0:
            return
        r = self._row(req, True)
        row = (self.key_rows if is_key else self.val_rows)[r]
        cap = self.capacity
        for x, slot in zip(values, slots):
            slot = int(slot)
            if slot in row.slots:
                row.data[row.slots.index(slot)] = np.asarray(x, F32)
                continue
            while row.length >= cap:
                self._flush(row, is_key, cap if is_key else 1)
            tail = (row.start + row.length) % cap
            row.slots[tail] = slot
            row.data[tail] = np.asarray(x, F32)
            row.length += 1

    def write_decode(self, reqs, key, value, slots):
        """``_write_kivi_cache`` with one token per request."""
        for i, req in enumerate(reqs):
            if int(slots[i]) < 0:
                continue
            self.store(req, key[i:i + 1], slots[i:i + 1], True)
            self.store(req, value[i:i + 1], slots[i:i + 1], False)

    def write_prefill(self, req, key, value, slots):
        """``_write_kivi_prefill_cache`` for one request's prompt."""
        keep = [i for i, s in enumerate(slots) if int(s) >= 0]
        key, value = key[keep], value[keep]
        slots = [int(slots[i]) for i in keep]
        n = len(slots)
        flush = (n // self.capacity) * self.capacity
        if flush:
            if not is_aligned_key_window(slots[:flush], self.group_size, self.block_size):
                raise RuntimeError("KIVI key flush requires contiguous aligned token groups.")
            self.flushes.append((True, slots[:flush], np.asarray(key[:flush], F32)))
            self.flushes.append((False, slots[:flush], np.asarray(value[:flush], F32)))
        if flush < n:
            self.store(req, key[flush:], slots[flush:], True)
            self.store(req, value[flush:], slots[flush:], False)

    def sync(self, reqs, block_table, seq_lens):
        """``_sync_kivi_residual_windows`` (:813-836): drop window slots the
        request no longer owns; the survivors are compacted to lanes 0.."""
        live = ordered_slots(block_table, seq_lens, self.block_size)
        for i, req in enumerate(reqs):
            r = self.req_to_row.get(req)
            if r is None:
                continue
            ls = set(live[i])
            for rows in (self.key_rows, self.val_rows):
                row = rows[r]
                lanes = self._lanes(row)
                keep = [l for l in lanes if row.slots[l] in ls]
                if len(keep) == len(lanes):
                    continue
                slots = [row.slots[l] for l in keep]
                data = [row.data[l] for l in keep]
                rows[r] = _Row(slots + [None] * (self.capacity - len(keep)),
                               data + [None] * (self.capacity - len(keep)), 0, len(keep))

    def apply_flushes(self, views):
        """Replays the recorded pack launches into six numpy views."""
        kq, ks, km, vq, vs, vm = views
        for is_key, slots, data in self.flushes:
            if is_key:
                kivi_pack_key(data, slots, kq, ks, km, self.group_size)
            else:
                kivi_pack_value(data, slots, vq, vs, vm, self.group_size)
        self.flushes = []
