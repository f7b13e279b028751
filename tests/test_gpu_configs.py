"""Attention parity at the benchmarked workloads.

Each test builds the workload exactly as ``bench.py`` does (same seeds,
shapes, outliers, block tables and cache state), runs the kernel the bench
times, and checks requests against the reference's CPU read path (the
oracle's numpy port): every request of the small configs, a seeded sample of
the large ones. The reference dequantises to the query dtype (bf16) before
attending; that variant is the one asserted, with the oracle's bound
(max-abs 1e-2, or one bf16 step of the reference value where bf16 cannot
resolve 1e-2). KIVI outputs are also held to the bound against the
fp32-dequantised variant (the KIVI decode kernel uses the exact dequantised
values)."""

from __future__ import annotations

import json

import pytest
import torch

import bench

pytestmark = pytest.mark.gpu


def dev():
    return torch.device("cuda", 0)


def _no_device_error():
    from qkv_b200.ops import _lib

    code = _lib.device_error(torch.cuda.current_stream().cuda_stream)
    assert code == 0, _lib.DEVICE_ERRORS.get(code, code)


def _assert(res, *variants):
    print(json.dumps(res))
    for v in variants:
        assert res[v]["within_bound"], (v, res[v])


def test_config1_int8_decode_every_request():
    from qkv_b200.ops import int8_paged_decode

    c = bench.build_config1(dev())
    out = torch.full_like(c.q, float("nan"))
    int8_paged_decode(c.q, c.kc, c.vc, c.k_aq, c.v_aq, c.bt_dev, c.seq_lens, c.D ** -0.5, out, max(c.lens))
    torch.cuda.synchronize()
    _assert(bench.cpu_check_int8(c, out, range(len(c.lens)), time_runs=0), "vs_bf16_cast")
    _no_device_error()


def test_config2_kivi_decode_every_request():
    from qkv_b200.ops import kivi_paged_decode

    c = bench.build_config2(dev())
    out = torch.full_like(c.q, float("nan"))
    kivi_paged_decode(c.q, c.views, c.rk, c.rv, c.bt_dev, c.seq_lens, c.state_dev, c.g, c.D ** -0.5, out,
                      max(c.lens))
    torch.cuda.synchronize()
    _assert(bench.cpu_check_kivi(c, out, range(len(c.lens)), time_runs=0), "vs_bf16_cast", "vs_fp32_dequant")
    _no_device_error()


def test_config3_int8_decode_full_shape_sampled():
    """64 x 8192 tokens, Hq 32 / KVH 8, block tables a permutation of the
    4096 physical blocks, 1% x16 outlier channels; 4 requests checked."""
    from qkv_b200.ops import int8_paged_decode

    w = bench.build_int8_workload(dict(bench.CONFIG3), 0, 1, dev())
    out = torch.full_like(w.q, float("nan"))
    int8_paged_decode(w.q, w.kc, w.vc, w.k_aq, w.v_aq, w.bt_dev, w.seq_lens, w.D ** -0.5, out, w.L)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    _assert(bench.cpu_check_int8(w, out, [0, 21, 42, 63], time_runs=0), "vs_bf16_cast")
    _no_device_error()


def test_config4_chunks_and_decode_rows_full_shape():
    """2 x 2048-token chunks over 6144 cached tokens (g 64) through the dense
    gather + tcgen05 prompt attention, and the 30 decode rows at
    U{2048..16384} through the paged decode kernel."""
    from qkv_b200.ops import dense_prefill, kivi_dequant_gather, kivi_paged_decode

    c = bench.build_config4(dict(bench.CONFIG4), dev())
    out_pre = torch.full_like(c.q_pre, float("nan"))
    out_dec = torch.full_like(c.q_dec, float("nan"))
    kivi_dequant_gather(c.views, c.rk, c.rv, c.bt_pre, c.kv_pre, c.st_pre, c.g, out_key=c.dk, out_value=c.dv,
                        cu_seqlens=c.cu_k_pre, seq_lens_device=c.len_pre)
    dense_prefill(c.q_pre, c.dk, c.dv, c.q_lens_pre, c.kv_pre, c.D ** -0.5, out_pre, causal=True,
                  cu_seqlens_q=c.cu_q_pre, cu_seqlens_k=c.cu_k_pre)
    kivi_paged_decode(c.q_dec, c.views, c.rk, c.rv, c.bt_dec, c.len_dec, c.st_dec, c.g, c.D ** -0.5, out_dec,
                      c.max_dec)
    torch.cuda.synchronize()
    assert torch.isfinite(out_pre.float()).all() and torch.isfinite(out_dec.float()).all()
    rows = [0, 1, 511, 777, 1500, c.q_lens_pre[0] - 1]
    _assert(bench.cpu_check_chunks(c, out_pre, rows), "vs_bf16_cast")
    dec = list(range(len(c.q_lens_pre), len(c.lens)))
    cd = bench.SimpleNamespace(views=c.views, rk=c.rk, rv=c.rv, bt=c.bt_dec, state=c.st_dec,
                               lens=[c.lens[b] for b in dec], q=c.q_dec, g=c.g, blk=c.blk, D=c.D)
    _assert(bench.cpu_check_kivi(cd, out_dec, [0, 7, 17, 29], time_runs=0), "vs_bf16_cast", "vs_fp32_dequant")
    _no_device_error()


def test_config5_kivi_decode_full_shape_sampled():
    """32 x 32768 tokens, Hq 64 / KVH 8, g 128 / r 128, x10 key outliers on 2%
    of (head, channel) pairs, caches built by bulk prefill + the window; 4
    requests checked."""
    from qkv_b200.ops import kivi_paged_decode

    w = bench.build_workload(dict(bench.CONFIG5), 0, 1, dev())
    out = torch.full((w.B, w.Hql, w.D), float("nan"), dtype=torch.bfloat16, device=dev())
    kivi_paged_decode(w.q, w.views, w.rk, w.rv, w.bt_dev, w.seq_lens, w.state, w.g, w.D ** -0.5, out, w.L)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    wc = bench.SimpleNamespace(views=w.views, rk=w.rk, rv=w.rv, bt=w.bt, state=w.state, lens=[w.L] * w.B, q=w.q,
                               g=w.g, blk=w.blk, D=w.D)
    _assert(bench.cpu_check_kivi(wc, out, [0, 10, 20, 31], time_runs=0), "vs_bf16_cast", "vs_fp32_dequant")
    _no_device_error()
