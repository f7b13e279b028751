"""FP8 per-token-head contract on CPU: the oracle against the reference's own
semantics (golden vectors), the byte layout against the reference's buffers,
and fail-closed layout derivation. No GPU."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import qkv_oracle as O
from conftest import bf16_to_f32
from qkv_b200.dtypes import KVQuantMode, get_kv_quant_mode, resolve_layout
from qkv_b200.methods.fp8_per_token_head.byte_cache import (
    Fp8PerTokenHeadLayout,
    fp8_caches_from_byte_tensors,
    fp8_per_token_head_layout,
)


def test_oracle_quantize_matches_reference_semantics(golden):
    g = golden("fp8")
    for side, codes, scale in (("key", "k_codes", "k_scale"), ("value", "v_codes", "v_scale")):
        q, s = O.fp8_quantize(bf16_to_f32(g[side]))
        assert np.array_equal(q, g[codes]), side
        assert np.array_equal(s.view(np.uint32), g[scale].view(np.uint32)), side
    q, s = O.fp8_quantize(bf16_to_f32(g["key"]))
    assert np.array_equal(O.fp8_dequantize(q, s).view(np.uint32), g["k_dequant"].view(np.uint32))
    qv, sv = O.fp8_quantize(bf16_to_f32(g["value"]))
    assert np.array_equal(O.bf16_round(O.fp8_dequantize(qv, sv)), g["v_fake"])


def test_zero_token_head_takes_the_scale_floor(golden):
    g = golden("fp8")
    assert g["k_scale"][5, 1, 0] == np.float32(1e-6)
    assert not g["k_codes"][5, 1].any()


def test_e4m3_encoder_matches_torch_on_every_code_and_midpoint():
    vals = np.unique(O.e4m3_decode(np.arange(256, dtype=np.uint8)))
    vals = vals[np.isfinite(vals)]
    mids = ((vals[1:].astype(np.float64) + vals[:-1]) / 2).astype(np.float32)
    xs = np.concatenate([vals, mids, np.nextafter(mids, np.float32(np.inf)), np.nextafter(mids, np.float32(-np.inf))])
    xs = np.clip(xs, -448, 448).astype(np.float32)
    want = torch.from_numpy(xs).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.e4m3_encode(xs), want)
    back = O.e4m3_decode(np.arange(256, dtype=np.uint8))
    torch_back = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    fin = np.isfinite(torch_back)
    assert np.array_equal(back[fin], torch_back[fin]) and np.isnan(back[~fin]).all()


def test_views_read_the_reference_buffers(golden):
    g = golden("fp8")
    T, H, D, blk, nb = g["geometry"].tolist()
    lay = Fp8PerTokenHeadLayout(num_blocks=nb, block_size=blk, num_kv_heads=H, head_size=D)
    kbuf, vbuf = torch.from_numpy(g["k_buffer"]), torch.from_numpy(g["v_buffer"])
    assert fp8_per_token_head_layout(kbuf, vbuf, num_kv_heads=H, head_size=D) == lay
    kd, ks, vd, vs = fp8_caches_from_byte_tensors(kbuf, vbuf, lay)
    slots = torch.from_numpy(g["slots"])
    assert np.array_equal(kd.view(nb * blk, H, D)[slots].numpy(), g["k_codes"])
    assert np.array_equal(vs.view(nb * blk, H, 1)[slots].numpy(), g["v_scale"])
    # oracle store through the same views writes the same bytes
    kb2, vb2 = torch.zeros_like(kbuf), torch.zeros_like(vbuf)
    v2 = [t.numpy() for t in fp8_caches_from_byte_tensors(kb2, vb2, lay)]
    O.fp8_store(bf16_to_f32(g["key"]), bf16_to_f32(g["value"]), g["slots"], *v2)
    assert np.array_equal(kb2.numpy(), g["k_buffer"]) and np.array_equal(vb2.numpy(), g["v_buffer"])


def test_layout_budget_and_fail_closed():
    lay = Fp8PerTokenHeadLayout(num_blocks=3, block_size=128, num_kv_heads=8, head_size=128)
    assert lay.bytes_per_token_head == 132 and lay.page_size_bytes() == 2 * 128 * 8 * 132
    assert lay.compression_vs_fp16() == pytest.approx(256 / 132)
    with pytest.raises(ValueError, match="divisible by 4"):
        Fp8PerTokenHeadLayout(num_blocks=1, block_size=16, num_kv_heads=1, head_size=30)
    k = torch.zeros(2, 16, 2, 36, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="equal regions"):
        fp8_per_token_head_layout(k, k[:1], num_kv_heads=2, head_size=32)
    with pytest.raises(RuntimeError, match="whole number of pages"):
        fp8_per_token_head_layout(k, k.clone(), num_kv_heads=2, head_size=36)
    with pytest.raises(RuntimeError, match="must hold"):
        fp8_caches_from_byte_tensors(k, k.clone(), Fp8PerTokenHeadLayout(num_blocks=2, block_size=8,
                                                                         num_kv_heads=2, head_size=32))


def test_dtype_contract():
    assert get_kv_quant_mode("fp8_per_token_head") is KVQuantMode.FP8_PER_TOKEN_HEAD
    assert int(KVQuantMode.FP8_PER_TOKEN_HEAD) == 10
    lay = resolve_layout("fp8_per_token_head", 128)
    assert lay.storage_dtype == "uint8" and lay.packed_last_dim == 128
    with pytest.raises(ValueError, match="divisible"):
        resolve_layout("fp8_per_token_head", 130)
