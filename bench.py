"""Benchmark of the quantized-KV decode hot path on B200.

Default workload: KIVI INT4 long-context decode,
32 requests at context 32768, 64 query / 8 KV heads, head 128, group 128,
residual 128, sharded by KV head across N GPUs (GPU i owns KV heads
[8i/N, 8(i+1)/N) and their query heads) with one NVLink peer all-gather of
the attention outputs per step (qkv_peer_combine_allgather, the split combine
fused into it). The cache of every request is built the way the
reference builds it — bulk prefill of L-1 tokens (floor(n/r)*r straight to
int4, the rest to the bf16 window) plus one decode write — with K/V ~ N(0,1)
in bf16 and x10 key outliers on 2% of (head, channel) pairs.

One step = one decode-attention pass of every request over its int4 pages and
bf16 windows (``qkv_kivi_paged_decode``: split-KV kernel + combine) followed,
for N > 1, by the all-gather. The caches (1.22 GB / N per GPU) exceed the
126 MB L2, so no L2 flush is needed between steps.

Reported on one JSON line (rank 0):
  value     tokens/s/layer over all GPUs, inputs resident in HBM, device-timed
            with CUDA events, max over ranks; the step is captured once as a
            CUDA graph (decode + combine; for N > 1 the combine runs fused
            with the NVLink peer all-gather of the heads,
            qkv_peer_combine_allgather) and replayed, as a serving loop does;
  roofline  algorithmic bytes per decode call / its CUDA-event time vs the
            measured HBM copy bandwidth (MEASURED_PEAKS.json);
  pack      KIVI pack GB/s (config 2 definition, 5248 B/token);
  e2e       the same metric through the plugin API — the KIVI mixin's
            ``forward()`` in DecodeOnly state with pinned host q/k/v copied in,
            the heads of all ranks gathered (N > 1) and the output copied out
            every step;
  cpu_baseline  the reference's CPU path (numpy port in oracle/) on a bounded
            sample of the workload, rank 0, N = 1 only.

``--impl reference`` times that CPU path alone (rank 0) on the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path
from types import SimpleNamespace

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "vllm-ascend-quantized-kv-cache-hust_b200"))

METRIC = "quantized-KV decode attn tokens/s/layer"
UNIT = "tokens/s/layer"

CONFIG5 = dict(batch=32, context=32768, num_heads=64, num_kv_heads=8, head_size=128, group_size=128,
               residual=128, block_size=128)
CONFIG2_PACK = dict(tokens=8192, num_kv_heads=8, head_size=128, group_size=128, block_size=128)
CONFIG3 = dict(batch=64, context=8192, num_heads=32, num_kv_heads=8, head_size=128, block_size=128)
CONFIG4 = dict(num_heads=32, num_kv_heads=8, head_size=128, group_size=64, residual=128, block_size=128,
               chunk=2048, cached=6144, prefills=2, decodes=30, decode_min=2048, decode_max=16384)


def parse():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--e2e-steps", type=int, default=200,
                    help="timed steps of the end-to-end leg (10 untimed first; at most 246), 0 skips it")
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the CPU legs (the oracle's port of the reference's CPU path: timed baseline and the "
                         "parity check of sampled requests)")
    ap.add_argument("--no-int8", action="store_true", help="skip the config-3 INT8 leg")
    ap.add_argument("--no-config4", action="store_true", help="skip the config-4 chunked-prefill leg")
    ap.add_argument("--shard", type=int, default=None,
                    help="with --only kivi: build rank 0's share of an N-way KV-head shard on this one GPU "
                         "(the per-GPU decode of an N-GPU run)")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the request count (small cases for ncu captures)")
    ap.add_argument("--only", choices=("kivi", "int8", "config4", "fp8", "small", "pack"), default=None,
                    help="run just one decode kernel loop (for ncu captures)")
    args = ap.parse_args()
    args.check = not args.no_cpu_baseline
    return args


# ---------------------------------------------------------------------------
# CPU path (the reference's algorithm, numpy port in oracle/)
# ---------------------------------------------------------------------------


def cpu_reference_sample(cfg, seed=0):
    """Builds one request of the workload on the host and returns a closure
    running the reference's CPU decode path on it: gather + dequantise the
    int4 history (kivi_dequant_gather_cache), overwrite the residual tail,
    fp32 attention (_forward_kivi_dense_attention)."""
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import qkv_oracle as O

    rng = np.random.default_rng(seed)
    L, H, D, g, blk, r = (cfg[k] for k in ("context", "num_kv_heads", "head_size", "group_size", "block_size",
                                           "residual"))
    Hq = cfg["num_heads"]
    pages = (L + blk - 1) // blk
    hist = ((L - 1) // r) * r  # bulk prefill of L-1 tokens flushes floor((L-1)/r)*r
    nbp = pages
    views = [
        np.zeros((nbp, H, D, blk // 8), np.int32), np.ones((nbp, H, D, blk // g), np.float32),
        np.zeros((nbp, H, D, blk // g), np.float32), np.zeros((nbp, blk, H, D // 8), np.int32),
        np.ones((nbp, blk, H, D // g), np.float32), np.zeros((nbp, blk, H, D // g), np.float32),
    ]
    # packed words / scales drawn directly (the CPU timing does not depend on
    # how they were produced)
    views[0][:] = rng.integers(-(2 ** 31), 2 ** 31 - 1, size=views[0].shape, dtype=np.int64).astype(np.int32)
    views[3][:] = rng.integers(-(2 ** 31), 2 ** 31 - 1, size=views[3].shape, dtype=np.int64).astype(np.int32)
    views[1][:] = rng.uniform(0.05, 0.5, views[1].shape)
    views[4][:] = rng.uniform(0.05, 0.5, views[4].shape)
    views[2][:] = rng.uniform(-3, 0, views[2].shape)
    views[5][:] = rng.uniform(-3, 0, views[5].shape)
    bt = rng.permutation(nbp).reshape(1, nbp)
    res = L - hist
    kwin = [O.bf16_round(rng.standard_normal((res, H, D)).astype(np.float32))]
    vwin = [O.bf16_round(rng.standard_normal((res, H, D)).astype(np.float32))]
    q = O.bf16_round(rng.standard_normal((1, Hq, D)).astype(np.float32))

    def run():
        dk, dv = O.kivi_dequant_gather(*views, bt, [L], g, target_bf16=True)
        dk, dv = O.overwrite_residual_tail(dk, dv, [L], kwin, vwin)
        return O.dense_attention(q, dk, dv, [1], [L], D ** -0.5, causal=True)

    return run


def _oracle():
    sys.path.insert(0, str(ROOT / "oracle"))
    import qkv_oracle as O

    return O


def kivi_sample(views, rk, rv, bt, state, lens, blk, reqs):
    """Host copies of what the reference's KIVI read path needs for requests
    ``reqs``: their pages of the six views (in block-table order, so the
    sample's block table is 0..n-1) and their key / value windows in FIFO
    order, as numpy arrays."""
    import torch

    bt = bt.cpu()
    st = state.cpu() if torch.is_tensor(state) else torch.tensor(state)
    cap = rk.shape[1]
    out = []
    for b in reqs:
        L = int(lens[b])
        n = (L + blk - 1) // blk
        pages = bt[b, :n].long()
        v = [x[pages.to(x.device)].cpu().numpy() for x in views]
        row, ks, kl, vs, vl, _ = (int(z) for z in st[b])

        def win(buf, start, length):
            if length <= 0:
                return None
            idx = ((start + torch.arange(length)) % cap).to(buf.device)
            return buf[row, idx].float().cpu().numpy()

        out.append((v, L, win(rk, ks, kl), win(rv, vs, vl)))
    return out


def cpu_check_kivi(c, out, reqs, time_runs=5, scale=None):
    """The reference's CPU read path (oracle/ numpy port) on requests
    ``reqs`` of a KIVI workload ``c`` (views, rk, rv, bt, state, lens, q, g,
    blk, D): its outputs against the GPU's ``out`` rows, with the dequantised
    K/V cast to bf16 as the reference casts them to the query dtype, and kept
    in fp32. With ``time_runs`` > 0 the bf16-cast path of the first sampled
    request is also timed (1 warm-up, then the median of ``time_runs``): the
    CPU baseline of the leg, in decode tokens/s/layer."""
    import numpy as np

    O = _oracle()
    reqs = list(reqs)
    scale = c.D ** -0.5 if scale is None else scale
    samples = kivi_sample(c.views, c.rk, c.rv, c.bt, c.state, c.lens, c.blk, reqs)
    q = c.q.float().cpu().numpy()
    got = out.float().cpu().numpy()
    res = {"requests": reqs}
    for name, cast in (("vs_bf16_cast", True), ("vs_fp32_dequant", False)):
        want = np.concatenate([
            O.kivi_decode_reference(v, np.arange((L + c.blk - 1) // c.blk, dtype=np.int32)[None], [L], [kw], [vw],
                                    q[b:b + 1], c.g, scale, target_bf16=cast)
            for b, (v, L, kw, vw) in zip(reqs, samples)])
        res[name] = O.attention_error(got[reqs], want)
    if time_runs > 0:
        v, L, kw, vw = samples[0]
        b = reqs[0]
        bt0 = np.arange((L + c.blk - 1) // c.blk, dtype=np.int32)[None]
        run = lambda: O.kivi_decode_reference(v, bt0, [L], [kw], [vw], q[b:b + 1], c.g, scale, target_bf16=True)
        res["cpu"] = _time_cpu(run, time_runs, f"request {b} (context {L})")
    return res


def cpu_check_int8(c, out, reqs, time_runs=5):
    """As ``cpu_check_kivi`` for an INT8 workload (kc, vc, k_aq, v_aq, bt,
    lens, q, blk, D): the reference's dense dequantisation (bf16 ``code *
    aq``, or kept in fp32) and fp32 attention."""
    import numpy as np

    O = _oracle()
    reqs = list(reqs)
    bt = c.bt.cpu()
    k_aq, v_aq = c.k_aq.float().cpu().numpy(), c.v_aq.float().cpu().numpy()
    q = c.q.float().cpu().numpy()
    got = out.float().cpu().numpy()
    samples = []
    for b in reqs:
        L = int(c.lens[b])
        pages = bt[b, :(L + c.blk - 1) // c.blk].long().to(c.kc.device)
        samples.append((c.kc[pages].cpu().numpy(), c.vc[pages].cpu().numpy(), L))
    res = {"requests": reqs}
    scale = c.D ** -0.5

    def ref(kc, vc, L, b, cast):
        bt0 = np.arange(kc.shape[0], dtype=np.int32)[None]
        return O.int8_decode_reference(kc, vc, k_aq, v_aq, bt0, [L], q[b:b + 1], scale, target_bf16=cast)

    for name, cast in (("vs_bf16_cast", True), ("vs_fp32_dequant", False)):
        want = np.concatenate([ref(kc, vc, L, b, cast) for b, (kc, vc, L) in zip(reqs, samples)])
        res[name] = O.attention_error(got[reqs], want)
    if time_runs > 0:
        kc, vc, L = samples[0]
        res["cpu"] = _time_cpu(lambda: ref(kc, vc, L, reqs[0], True), time_runs,
                               f"request {reqs[0]} (context {L})")
    return res


def _time_cpu(run, runs, what):
    """1 warm-up, then the median of ``runs`` timed calls: decode tokens/s/layer
    of one request (one query token per call)."""
    run()
    times = []
    for _ in range(runs):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": 1.0 / t, "unit": UNIT, "seconds_per_request": t, "runs": runs, "sample": what,
            **cpu_info()}


def cpu_info() -> dict:
    """Host CPU model, logical cores and the BLAS / torch thread counts the
    numpy port runs with."""
    model = ""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    try:
        import torch

        torch_threads = torch.get_num_threads()
    except Exception:
        torch_threads = None
    return {"cpu_model": model, "cpu_count": os.cpu_count(), "cores": cpu_threads(),
            "torch_threads": torch_threads}


def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 1) for i in threadpool_info()]
        return max(n) if n else 1
    except Exception:
        return 1


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = CONFIG5
    run = cpu_reference_sample(cfg)
    for _ in range(max(args.warmup, 0)):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    value = 1.0 / dt  # one decode token of one request per step
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int4/bf16->fp32",
        "data": "synthetic",
        "config": workload_config(cfg, args.gpus),
        "cpu_baseline": {
            "value": value, "unit": UNIT, "kind": "port",
            "sample": "one request of the workload per step (context 32768, 64 q / 8 kv heads); the CPU path is "
                      "linear in requests, so tokens/s/layer of the sample is that of the full batch",
            **cpu_info(),
        },
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(cfg, n):
    return {
        "workload": "BASELINE config 5: KIVI INT4 long-context decode, KV-head sharded",
        "batch": cfg["batch"], "context": cfg["context"], "num_heads": cfg["num_heads"],
        "num_kv_heads": cfg["num_kv_heads"], "head_size": cfg["head_size"], "group_size": cfg["group_size"],
        "residual": cfg["residual"], "block_size": cfg["block_size"],
        "parallelism": f"kv-head shard x{n}" + (" + NVLink peer all-gather" if n > 1 else ""),
        "l2": "inputs larger than L2 (KIVI cache 1.22 GB / N per GPU), no flush",
    }


# ---------------------------------------------------------------------------
# GPU build of the workload
# ---------------------------------------------------------------------------


def build_workload(cfg, rank, world, device, seed=1234):
    """Per-rank KIVI caches + windows of config 5, built with the pack kernels
    following the reference's bulk-prefill + one-decode-write semantics."""
    import torch

    from qkv_b200.methods.kivi_int4.byte_cache import KiviByteCacheLayout, kivi_caches_from_byte_tensors
    from qkv_b200.ops import kivi_pack_key_cache, kivi_pack_value_cache

    B, L, Hq, H, D, g, r, blk = (cfg[k] for k in ("batch", "context", "num_heads", "num_kv_heads", "head_size",
                                                 "group_size", "residual", "block_size"))
    assert H % world == 0 and Hq % world == 0
    Hl, Hql = H // world, Hq // world
    pages = (L + blk - 1) // blk
    spare = 2  # pages per request for e2e steps beyond the context
    nb = B * (pages + spare)
    gen = torch.Generator(device=device).manual_seed(seed)
    cpu_gen = torch.Generator().manual_seed(seed)
    lay = KiviByteCacheLayout(num_blocks=nb, block_size=blk, num_kv_heads=Hl, head_size=D, group_size=g)
    kbuf = torch.zeros(nb, blk, Hl, lay.bytes_per_token_head, dtype=torch.uint8, device=device)
    vbuf = torch.zeros_like(kbuf)
    views = kivi_caches_from_byte_tensors(kbuf, vbuf, lay)
    perm = torch.randperm(nb, generator=cpu_gen)
    bt = perm.view(B, pages + spare).to(torch.int32)
    # key outliers: x10 on 2% of (head, channel) pairs of the FULL model; this
    # rank keeps its heads' share
    n_out = max(1, int(0.02 * H * D))
    out_idx = torch.randperm(H * D, generator=cpu_gen)[:n_out]
    kscale = torch.ones(H * D)
    kscale[out_idx] = 10.0
    kscale = kscale.view(H, D)[rank * Hl:(rank + 1) * Hl].to(device)
    hist = ((L - 1) // r) * r
    res = L - hist
    rk = torch.zeros(B + 1, r, Hl, D, dtype=torch.bfloat16, device=device)
    rv = torch.zeros_like(rk)
    pos = torch.arange(L, device=device)
    for b in range(B):
        k = (torch.randn(L, Hl, D, generator=gen, device=device) * kscale).to(torch.bfloat16)
        v = torch.randn(L, Hl, D, generator=gen, device=device).to(torch.bfloat16)
        slots = bt[b].to(device).long()[pos // blk] * blk + pos % blk
        kivi_pack_key_cache(k[:hist].contiguous(), slots[:hist].contiguous(), *views[:3], g, validate_slots=False)
        kivi_pack_value_cache(v[:hist].contiguous(), slots[:hist].contiguous(), *views[3:], g)
        rk[b, :res] = k[hist:]
        rv[b, :res] = v[hist:]
    torch.cuda.synchronize(device)
    q = torch.randn(B, Hql, D, generator=gen, device=device).to(torch.bfloat16)
    # window state of request b: row b, start 0, both windows = the last `res` positions
    state = torch.tensor([[b, 0, res, 0, res, L] for b in range(B)], dtype=torch.int32, device=device)
    return SimpleNamespace(
        views=views, kbuf=kbuf, vbuf=vbuf, layout=lay, bt=bt, bt_dev=bt.to(device), rk=rk, rv=rv, q=q,
        state=state, seq_lens=torch.full((B,), L, dtype=torch.int32, device=device), hist=hist, res=res,
        B=B, L=L, Hl=Hl, Hql=Hql, D=D, g=g, r=r, blk=blk, nb=nb, pages=pages,
    )


def build_kivi_requests(lens, H, D, g, r, blk, device, cpu_gen, gen, outlier_frac=0.02, factor=10.0):
    """KIVI caches of requests with the given lengths in the state the
    reference's writes leave: int4 history of the first ``((L - 1) // r) * r``
    positions packed through ``kivi_pack_*`` over a permuted block table, the
    rest in the bf16 windows (row b = request b). K/V ~ N(0,1) bf16 with
    ``factor`` x key outliers on ``outlier_frac`` of (head, channel) pairs."""
    import torch

    from qkv_b200.methods.kivi_int4.byte_cache import KiviByteCacheLayout, kivi_caches_from_byte_tensors
    from qkv_b200.ops import kivi_pack_key_cache, kivi_pack_value_cache

    B = len(lens)
    pages = [(L + blk - 1) // blk for L in lens]
    maxp = max(pages)
    nb = sum(pages) + 1
    lay = KiviByteCacheLayout(num_blocks=nb, block_size=blk, num_kv_heads=H, head_size=D, group_size=g)
    kbuf = torch.zeros(nb, blk, H, lay.bytes_per_token_head, dtype=torch.uint8, device=device)
    vbuf = torch.zeros_like(kbuf)
    views = kivi_caches_from_byte_tensors(kbuf, vbuf, lay)
    perm = torch.randperm(nb, generator=cpu_gen)
    bt = torch.zeros(B, maxp, dtype=torch.int32)
    kscale = torch.ones(H * D)
    kscale[torch.randperm(H * D, generator=cpu_gen)[:max(1, int(outlier_frac * H * D))]] = factor
    kscale = kscale.view(H, D).to(device)
    rk = torch.zeros(B + 1, r, H, D, dtype=torch.bfloat16, device=device)
    rv = torch.zeros_like(rk)
    state = []
    cur = 0
    for b, L in enumerate(lens):
        bt[b, :pages[b]] = perm[cur:cur + pages[b]].to(torch.int32)
        cur += pages[b]
        hist = ((L - 1) // r) * r
        res = L - hist
        k = (torch.randn(L, H, D, generator=gen, device=device) * kscale).to(torch.bfloat16)
        v = torch.randn(L, H, D, generator=gen, device=device).to(torch.bfloat16)
        pos = torch.arange(L, device=device)
        slots = bt[b].to(device).long()[pos // blk] * blk + pos % blk
        if hist:
            kivi_pack_key_cache(k[:hist].contiguous(), slots[:hist].contiguous(), *views[:3], g,
                                validate_slots=False)
            kivi_pack_value_cache(v[:hist].contiguous(), slots[:hist].contiguous(), *views[3:], g)
        rk[b, :res] = k[hist:]
        rv[b, :res] = v[hist:]
        state.append([b, 0, res, 0, res, L])
    torch.cuda.synchronize(device)
    return SimpleNamespace(views=views, rk=rk, rv=rv, bt=bt, state=torch.tensor(state, dtype=torch.int32),
                           kbuf=kbuf, vbuf=vbuf)


def build_config4(cfg, device, seed=1004):
    """Config 4 (chunked prefill mixed with decode, KIVI g 64): 2 requests
    whose 2048-token chunk lands on 6144 cached tokens (history 8192 after the
    chunk's write) and 30 decode requests at L ~ U{2048..16384}, every cache
    in the state the reference's writes leave (int4 history + bf16 window),
    K/V ~ N(0,1) bf16 with x10 key outliers on 2% of (head, channel) pairs."""
    import torch

    Hq, H, D, g, r, blk = (cfg[k] for k in ("num_heads", "num_kv_heads", "head_size", "group_size", "residual",
                                           "block_size"))
    cpu_gen = torch.Generator().manual_seed(seed)
    gen = torch.Generator(device=device).manual_seed(seed)
    lens = [cfg["cached"] + cfg["chunk"]] * cfg["prefills"] + torch.randint(
        cfg["decode_min"], cfg["decode_max"] + 1, (cfg["decodes"],), generator=cpu_gen).tolist()
    B = len(lens)
    kv = build_kivi_requests(lens, H, D, g, r, blk, device, cpu_gen, gen)
    views, rk, rv, bt = kv.views, kv.rk, kv.rv, kv.bt
    state = kv.state.tolist()
    torch.cuda.synchronize(device)
    P, C = cfg["prefills"], cfg["chunk"]
    # query token i of a chunk attends to its causal length
    rows_len = [lens[b] - C + i + 1 for b in range(P) for i in range(C)]
    dec = list(range(P, B))
    st = torch.tensor(state, dtype=torch.int32)
    kv_pre = lens[:P]
    cu = lambda ns: torch.tensor([0] + torch.tensor(ns).cumsum(0).tolist(), dtype=torch.int32, device=device)
    return SimpleNamespace(
        views=views, rk=rk, rv=rv, g=g, D=D, H=H, Hq=Hq, blk=blk, lens=lens,
        # chunk requests: dense K/V gathered from int4 pages + windows, then
        # prompt attention aligned to the end of each request's keys
        q_pre=torch.randn(P * C, Hq, D, generator=gen, device=device).to(torch.bfloat16),
        q_lens_pre=[C] * P, kv_pre=kv_pre, cu_q_pre=cu([C] * P), cu_k_pre=cu(kv_pre),
        bt_pre=bt[:P].to(device), len_pre=torch.tensor(kv_pre, dtype=torch.int32, device=device),
        st_pre=st[:P].to(device),
        dk=torch.empty(sum(kv_pre), H, D, dtype=torch.bfloat16, device=device),
        dv=torch.empty(sum(kv_pre), H, D, dtype=torch.bfloat16, device=device),
        q_dec=torch.randn(len(dec), Hq, D, generator=gen, device=device).to(torch.bfloat16),
        bt_dec=bt[dec].to(device), len_dec=torch.tensor([lens[b] for b in dec], dtype=torch.int32, device=device),
        st_dec=st[dec].to(device), max_dec=max(lens[b] for b in dec),
        # work: 2 FLOP per multiply-add, QK and PV, every prefill row over its causal length
        prefill_flops=4 * Hq * D * sum(rows_len),
        # gather: int4 codes + group scale/min read (history), bf16 window
        # read, bf16 dense K and V written
        gather_bytes=sum(gather_bytes(L, H, D, g, r) for L in kv_pre),
        decode_bytes=sum(request_decode_bytes(lens[b], H, Hq, D, g, r, blk) for b in dec),
    )


def gather_bytes(L, H, D, g, r):
    """Algorithmic bytes of one request's dense gather: the int4 history with
    its per-group scale/min on both sides, the bf16 windows, and the bf16
    dense K and V written."""
    hist = ((L - 1) // r) * r
    res = L - hist
    return H * (2 * hist * (D // 2 + 8 * D // g) + 2 * res * D * 2 + 2 * L * D * 2)


def request_decode_bytes(L, H, Hq, D, g, r, blk):
    """Algorithmic bytes of one request's decode attention: int4 codes and
    per-group scale/min of the history on both sides, the bf16 windows, q,
    out and the block-table row."""
    hist = ((L - 1) // r) * r
    res = L - hist
    return H * (2 * hist * (D // 2 + 8 * D // g) + 2 * res * D * 2) + 2 * Hq * D * 2 + 4 * ((L + blk - 1) // blk)


def run_config4_leg(device, args):
    """Config 4 through the path the mixin takes (ChunkedPrefill with
    history): the chunk requests gather dense K/V from the int4 pages and the
    windows and run the tcgen05 prompt attention; the decode rows run the
    paged decode kernel. TFLOP/s of the prompt attention against the measured
    bf16 tensor peak, GB/s of the gather and the decode rows against HBM."""
    import torch

    from qkv_b200.ops import dense_prefill, kivi_dequant_gather, kivi_paged_decode

    c = build_config4(CONFIG4, device)
    out_pre = torch.empty_like(c.q_pre)
    out_dec = torch.empty_like(c.q_dec)
    sc = c.D ** -0.5

    def gather():
        kivi_dequant_gather(c.views, c.rk, c.rv, c.bt_pre, c.kv_pre, c.st_pre, c.g, out_key=c.dk, out_value=c.dv,
                            cu_seqlens=c.cu_k_pre, seq_lens_device=c.len_pre)

    def attend():
        dense_prefill(c.q_pre, c.dk, c.dv, c.q_lens_pre, c.kv_pre, sc, out_pre, causal=True,
                      cu_seqlens_q=c.cu_q_pre, cu_seqlens_k=c.cu_k_pre)

    def prefill():
        gather()
        attend()

    def decode():
        kivi_paged_decode(c.q_dec, c.views, c.rk, c.rv, c.bt_dec, c.len_dec, c.st_dec, c.g, sc, out_dec, c.max_dec)

    def step():
        prefill()
        decode()

    parity = None
    if args.check:
        step()
        torch.cuda.synchronize(device)
        dec = list(range(len(c.q_lens_pre), len(c.lens)))
        cd = SimpleNamespace(views=c.views, rk=c.rk, rv=c.rv, bt=c.bt_dec, state=c.st_dec,
                             lens=[c.lens[b] for b in dec], q=c.q_dec, g=c.g, blk=c.blk, D=c.D)
        parity = {"decode_rows": cpu_check_kivi(cd, out_dec, [0, 17], time_runs=0),
                  "chunk_rows": cpu_check_chunks(c, out_pre, [0, 1, 777, c.q_lens_pre[0] - 1])}
    steps = max(3, min(args.steps, 50))
    ms_gather = time_loop(gather, steps, 3, device)
    ms_attn = time_loop(attend, steps, 3, device)
    ms_pre = time_loop(prefill, steps, 3, device)
    ms_dec = time_loop(decode, args.steps, args.warmup, device)
    ms_step = time_loop(step, steps, 3, device)
    peaks = measured_peaks()
    tf_peak = peaks.get("bf16_tflops") or 1590.0
    hbm = peaks.get("hbm_gbs") or 6650.0
    tflops = c.prefill_flops / (ms_attn * 1e-3) / 1e12
    gbs = c.decode_bytes / (ms_dec * 1e-3) / 1e9
    gather_gbs = c.gather_bytes / (ms_gather * 1e-3) / 1e9
    tokens = len(c.q_lens_pre) * c.q_lens_pre[0] + c.q_dec.shape[0]
    return {"workload": "BASELINE config 4: 2 x 2048-token chunks on 6144 cached + 30 decodes, KIVI g 64, Hq 32 / KVH 8",
            "step_ms": ms_step, "step_tokens": tokens, "step_tokens_per_s": tokens / (ms_step * 1e-3),
            "prefill_ms": ms_pre, "prefill_path": "qkv_kivi_dequant_gather + tcgen05 qkv_dense_prefill",
            "gather_ms": ms_gather, "gather_bytes": c.gather_bytes, "gather_gbs": gather_gbs,
            "gather_frac_of_hbm": gather_gbs / hbm,
            "attn_ms": ms_attn, "prefill_flops": c.prefill_flops, "prefill_tflops": tflops,
            "prefill_frac_of_bf16_peak": tflops / tf_peak,
            "decode_ms": ms_dec, "decode_bytes": c.decode_bytes, "decode_gbs": gbs, "decode_frac_of_hbm": gbs / hbm,
            "parity": parity}


def cpu_check_chunks(c, out_pre, rows):
    """Prompt rows of config 4's chunk requests against the reference's
    generic branch (methods/kivi_int4/attention_backend.py:1157-1191): dense
    K/V from the int4 pages and the windows (cast to bf16, or kept in fp32),
    then fp32 attention of query row i over keys [0, L - chunk + i]."""
    import numpy as np

    O = _oracle()
    P = len(c.q_lens_pre)
    C = c.q_lens_pre[0]
    samples = kivi_sample(c.views, c.rk, c.rv, c.bt_pre, c.st_pre, c.kv_pre, c.blk, range(P))
    q = c.q_pre.float().cpu().numpy()
    got = out_pre.float().cpu().numpy()
    res = {"rows": rows, "requests": P}
    scale = c.D ** -0.5
    for name, cast in (("vs_bf16_cast", True), ("vs_fp32_dequant", False)):
        want, have = [], []
        for p, (v, L, kw, vw) in enumerate(samples):
            bt0 = np.arange((L + c.blk - 1) // c.blk, dtype=np.int32)[None]
            dk, dv = O.kivi_dequant_gather(*v, bt0, [L], c.g, target_bf16=cast)
            dk, dv = O.overwrite_residual_tail(dk, dv, [L], [kw], [vw])
            for i in rows:
                n = L - C + i + 1
                r = p * C + i
                want.append(O.dense_attention(q[r:r + 1], dk[:n], dv[:n], [1], [n], scale, causal=True))
                have.append(got[r:r + 1])
        res[name] = O.attention_error(np.concatenate(have), np.concatenate(want))
    return res


def run_small_configs(device, args):
    """Configs 1 and 2 (1 GPU): the small, latency-bound decode steps of
    BASELINE.json. Config 1: INT8, 4 requests at 512 / 1024 / 1536 / 2048,
    Hq 32 / KVH 8, K/V ~ N(0,1) with 4 fixed channels per head x20, scales
    from the four prompts as one prefill batch. Config 2: KIVI INT4, 8
    requests at L ~ U{1024..8192}, Hq 40 / KVH 8 (5 query heads per KV head),
    g 128, r 128, keys with x10 outliers on 2% of (head, channel) pairs. Each
    decode step is replayed from a CUDA graph and timed with CUDA events; both
    caches fit in L2, so L2 is flushed before every timed step."""
    import torch

    from qkv_b200.ops import int8_paged_decode, kivi_paged_decode

    peak = measured_peaks().get("hbm_gbs") or 6650.0
    out = {}
    # ---- config 1
    c1 = build_config1(device)
    D, H, Hq, blk, lens = c1.D, c1.H, c1.Hq, c1.blk, c1.lens
    o = torch.empty_like(c1.q)

    def dec1():
        int8_paged_decode(c1.q, c1.kc, c1.vc, c1.k_aq, c1.v_aq, c1.bt_dev, c1.seq_lens, D ** -0.5, o, max(lens))

    dec1()
    parity1 = cpu_check_int8(c1, o, range(len(lens)), time_runs=0) if args.check else None
    ms = time_loop_flushed(dec1, args.steps, args.warmup, device)
    pages = [(L + blk - 1) // blk for L in lens]
    by = sum(L * H * D * 2 for L in lens) + 2 * H * D * 2 + 2 * len(lens) * Hq * D * 2 + 4 * sum(pages)
    out["config1"] = {"workload": "BASELINE config 1: INT8, 4 requests at 512/1024/1536/2048, Hq 32 / KVH 8",
                      "ms_per_step": ms, "tokens_per_s_per_layer": len(lens) / (ms * 1e-3), "bytes_per_launch": by,
                      "hbm_gbs": by / (ms * 1e-3) / 1e9, "frac_of_measured_hbm": by / (ms * 1e-3) / 1e9 / peak,
                      "l2": "flushed: 256 MB written, then another 256 MB read, before every timed step", "parity": parity1}
    # ---- config 2
    c2 = build_config2(device)
    o = torch.empty_like(c2.q)

    def dec2():
        kivi_paged_decode(c2.q, c2.views, c2.rk, c2.rv, c2.bt_dev, c2.seq_lens, c2.state_dev, c2.g, c2.D ** -0.5, o,
                          max(c2.lens))

    dec2()
    parity2 = cpu_check_kivi(c2, o, range(len(c2.lens)), time_runs=0) if args.check else None
    ms = time_loop_flushed(dec2, args.steps, args.warmup, device)
    by = sum(request_decode_bytes(L, c2.H, c2.Hq, c2.D, c2.g, c2.r, c2.blk) for L in c2.lens)
    out["config2"] = {"workload": "BASELINE config 2: KIVI INT4 decode, 8 requests at U{1024..8192}, Hq 40 / KVH 8",
                      "lens": c2.lens, "ms_per_step": ms, "tokens_per_s_per_layer": len(c2.lens) / (ms * 1e-3),
                      "bytes_per_launch": by, "hbm_gbs": by / (ms * 1e-3) / 1e9,
                      "frac_of_measured_hbm": by / (ms * 1e-3) / 1e9 / peak,
                      "l2": "flushed: 256 MB written, then another 256 MB read, before every timed step", "parity": parity2}
    return out


def build_config1(device, seed=1001):
    """Config 1: INT8, 4 requests at 512 / 1024 / 1536 / 2048, Hq 32 / KVH 8,
    head 128, block 128; K/V ~ N(0,1) bf16 with 4 fixed channels per head
    x20; scales from the four prompts as one prefill batch, then every token
    quantised into the pages through a permuted block table."""
    import torch

    from qkv_b200.ops import int8_calc_scales, int8_quant_store

    gen = torch.Generator(device=device).manual_seed(seed)
    cpu_gen = torch.Generator().manual_seed(seed)
    lens, Hq, H, D, blk = [512, 1024, 1536, 2048], 32, 8, 128, 128
    scale = torch.ones(H, D)
    for h in range(H):
        scale[h, torch.randperm(D, generator=cpu_gen)[:4]] = 20.0
    scale = scale.to(device)
    T = sum(lens)
    k = (torch.randn(T, H, D, generator=gen, device=device) * scale).to(torch.bfloat16)
    v = (torch.randn(T, H, D, generator=gen, device=device) * scale).to(torch.bfloat16)
    k_inv, v_inv, k_aq, v_aq = int8_calc_scales(k, v)
    pages = [(L + blk - 1) // blk for L in lens]
    nb = sum(pages)
    bt = torch.zeros(len(lens), max(pages), dtype=torch.int32)
    perm = torch.randperm(nb, generator=cpu_gen).to(torch.int32)
    cur, slots = 0, []
    for b, L in enumerate(lens):
        bt[b, :pages[b]] = perm[cur:cur + pages[b]]
        cur += pages[b]
        slots += [int(bt[b, p // blk]) * blk + p % blk for p in range(L)]
    kc = torch.zeros(nb, blk, H, D, dtype=torch.int8, device=device)
    vc = torch.zeros_like(kc)
    int8_quant_store(k, v, torch.tensor(slots, device=device), k_inv, v_inv, kc, vc)
    q = torch.randn(len(lens), Hq, D, generator=gen, device=device).to(torch.bfloat16)
    return SimpleNamespace(kc=kc, vc=vc, k_aq=k_aq, v_aq=v_aq, bt=bt, bt_dev=bt.to(device), q=q, lens=lens,
                           seq_lens=torch.tensor(lens, dtype=torch.int32, device=device), H=H, Hq=Hq, D=D, blk=blk,
                           k=k, v=v, slots=slots)


def build_config2(device, seed=1002):
    """Config 2: KIVI INT4, 8 requests at L ~ U{1024..8192}, Hq 40 / KVH 8,
    head 128, g 128, r 128, keys x10 on 2% of (head, channel) pairs."""
    import torch

    gen = torch.Generator(device=device).manual_seed(seed)
    cpu_gen = torch.Generator().manual_seed(seed)
    Hq, H, D, g, r, blk = 40, 8, 128, 128, 128, 128
    lens = torch.randint(1024, 8193, (8,), generator=cpu_gen).tolist()
    kv = build_kivi_requests(lens, H, D, g, r, blk, device, cpu_gen, gen)
    q = torch.randn(len(lens), Hq, D, generator=gen, device=device).to(torch.bfloat16)
    return SimpleNamespace(views=kv.views, rk=kv.rk, rv=kv.rv, bt=kv.bt, bt_dev=kv.bt.to(device), state=kv.state,
                           state_dev=kv.state.to(device), q=q, lens=lens,
                           seq_lens=torch.tensor(lens, dtype=torch.int32, device=device), H=H, Hq=Hq, D=D, g=g, r=r,
                           blk=blk)


def build_int8_workload(cfg, rank, world, device, seed=4321):
    """Config 3 on this rank's KV heads: 64 requests x 8192 tokens in int8
    pages (block tables a permutation of the physical blocks), K/V ~ N(0,1)
    with x16 outliers on 1% of (head, channel) pairs, scales calibrated on the
    first request's K/V (the first batch a layer sees), then quantised."""
    import torch

    from qkv_b200.ops import int8_calc_scales, int8_quant_store

    B, L, Hq, H, D, blk = (cfg[k] for k in ("batch", "context", "num_heads", "num_kv_heads", "head_size",
                                           "block_size"))
    Hl, Hql = H // world, Hq // world
    pages = L // blk
    nb = B * pages
    gen = torch.Generator(device=device).manual_seed(seed)
    cpu_gen = torch.Generator().manual_seed(seed)
    n_out = max(1, int(0.01 * H * D))
    scale = torch.ones(H * D)
    scale[torch.randperm(H * D, generator=cpu_gen)[:n_out]] = 16.0
    scale = scale.view(H, D)[rank * Hl:(rank + 1) * Hl].to(device)
    bt = torch.randperm(nb, generator=cpu_gen).view(B, pages).to(torch.int32)
    kc = torch.empty(nb, blk, Hl, D, dtype=torch.int8, device=device)
    vc = torch.empty_like(kc)
    pos = torch.arange(L, device=device)
    k_inv = v_inv = k_aq = v_aq = None
    for b in range(B):
        k = (torch.randn(L, Hl, D, generator=gen, device=device) * scale).to(torch.bfloat16)
        v = (torch.randn(L, Hl, D, generator=gen, device=device) * scale).to(torch.bfloat16)
        if k_inv is None:
            k_inv, v_inv, k_aq, v_aq = int8_calc_scales(k, v)
        slots = bt[b].to(device).long()[pos // blk] * blk + pos % blk
        int8_quant_store(k, v, slots, k_inv, v_inv, kc, vc)
    torch.cuda.synchronize(device)
    q = torch.randn(B, Hql, D, generator=gen, device=device).to(torch.bfloat16)
    return SimpleNamespace(kc=kc, vc=vc, k_aq=k_aq, v_aq=v_aq, bt=bt, bt_dev=bt.to(device), q=q, lens=[L] * B,
                           seq_lens=torch.full((B,), L, dtype=torch.int32, device=device),
                           B=B, L=L, Hl=Hl, Hql=Hql, D=D, blk=blk)


def int8_bytes(w) -> int:
    """int8 K and V of every live token, the bf16 antiquant scales, q, out
    and the block table."""
    return w.B * (w.Hl * w.L * w.D * 2 + 2 * w.Hql * w.D * 2 + 4 * (w.L // w.blk)) + 2 * w.Hl * w.D * 2


def time_loop(fn, steps, warmup, device):
    """ms per call of ``fn`` replayed from a CUDA graph (captured after the
    warm-up calls), timed with CUDA events."""
    import torch

    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(max(warmup, 3)):
            fn()
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    graph.replay()
    torch.cuda.synchronize(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        graph.replay()
    e.record()
    torch.cuda.synchronize(device)
    del graph
    return s.elapsed_time(e) / steps


def time_loop_flushed(fn, steps, warmup, device):
    """ms per call of ``fn`` for workloads that fit in L2: before every timed
    replay a 256 MB buffer (twice the 126 MB L2) is written and a second
    256 MB buffer is read, and only the replay itself sits between that
    step's CUDA events. The read evicts the written lines, so their write-back
    to HBM happens before the timed replay and the L2 it starts from holds
    clean lines of neither the workload nor the flush (the state ncu's cache
    control gives a profiled launch); with the write alone, up to 126 MB of
    dirty flush lines would be written back during the timed replay."""
    import torch

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    clean = torch.zeros(32 << 20, dtype=torch.int64, device=device)
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(max(warmup, 3)):
            fn()
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    graph.replay()
    torch.cuda.synchronize(device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for s, e in ev:
        flush.zero_()
        clean.sum()
        s.record()
        graph.replay()
        e.record()
    torch.cuda.synchronize(device)
    del graph
    return sum(s.elapsed_time(e) for s, e in ev) / steps


def algorithmic_bytes(w) -> int:
    """Bytes one decode call must move: int4 codes + per-group scale/min of
    the history (keys: per channel per token group; values: per token per
    dim group), the bf16 windows, q, out and the block table."""
    B, L, H, Hq, D, g = w.B, w.L, w.Hl, w.Hql, w.D, w.g
    hk = hv = w.hist
    per_head = hk * D // 2 + (hk // g) * D * 8 + hv * D // 2 + hv * (D // g) * 8 + 2 * w.res * D * 2
    return B * (H * per_head + 2 * Hq * D * 2 + 4 * ((L + w.blk - 1) // w.blk))


_CLOCK_POLLER = r"""
import sys, time
idx, uuid, period = int(sys.argv[1]), sys.argv[2], float(sys.argv[3])
try:
    import pynvml as nv
    nv.nvmlInit()
    try:
        h = nv.nvmlDeviceGetHandleByUUID(uuid)
    except Exception:
        h = nv.nvmlDeviceGetHandleByIndex(idx)
    flags = [nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
             nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap]
    while True:
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        print(f"{sm},{mx},,{hex(r)}," + ",".join("Active" if r & f else "Not Active" for f in flags), flush=True)
        time.sleep(period)
except Exception:  # no NVML: nvidia-smi, slower
    import subprocess
    q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    while True:
        out = subprocess.run(["nvidia-smi", "--query-gpu=" + q, "--format=csv,noheader,nounits", "-i", str(idx)],
                             capture_output=True, text=True, timeout=5).stdout.strip()
        if out:
            print(out, flush=True)
        time.sleep(0.05)
"""


class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU during a region with
    read-only NVML queries every few milliseconds (nvidia-smi when NVML is
    missing). The poller is a child process, so the sampling rate does not
    depend on the benchmark's own Python thread; the region starts only after
    the first sample has arrived."""

    PERIOD_S = 0.003

    def __init__(self, index: int) -> None:
        self.index = index
        self.rows: list[list[str]] = []
        self._proc = None
        self._reader: threading.Thread | None = None
        self._first = threading.Event()
        self.uuid = ""
        try:
            import torch

            u = str(torch.cuda.get_device_properties(index).uuid)
            self.uuid = u if u.startswith("GPU-") else "GPU-" + u
        except Exception:
            pass

    def _read(self):
        for line in self._proc.stdout:
            self.rows.append([c.strip() for c in line.strip().split(",")])
            self._first.set()
        self._first.set()

    def __enter__(self):
        try:
            self._proc = subprocess.Popen(
                [sys.executable, "-c", _CLOCK_POLLER, str(self.index), self.uuid, str(self.PERIOD_S)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._reader = threading.Thread(target=self._read, daemon=True)
            self._reader.start()
            self._first.wait(timeout=60)
        except Exception:
            self._proc = None
        return self

    def __exit__(self, *exc):
        if self._proc is not None:
            self._proc.terminate()  # the poller this object started, by its own handle
            try:
                self._proc.wait(timeout=10)
            except Exception:
                self._proc.kill()
        if self._reader is not None:
            self._reader.join(timeout=10)

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for row in self.rows:
            try:
                sm.append(float(row[0]))
                mx = float(row[1])
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, row[4:8]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def profiled_traffic(name: str, world: int) -> int | None:
    """DRAM bytes (read + write) of one launch of the dominant kernel, from
    the committed ncu summary ``profiles/<name>`` (its
    ``traffic_bytes_per_launch:`` line, captured on one GPU); a rank of an
    N-GPU run holds 1/N of the heads, so its launch moves 1/N of them."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return int(line.split(":", 1)[1]) // max(world, 1)
    return None


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text())
    return {}


def bench_pack(device, check=False, tokens=None):
    """Pack GB/s (config 2's definition: 5248 B/token = 4096 bf16 in + 1152
    out at KVH 8, D 128, g 128): keys and values of 8192 tokens (or
    ``tokens``), one bulk-prompt flush of both sides."""
    import torch

    from qkv_b200.ops import kivi_pack_kv_cache

    c = CONFIG2_PACK
    T, H, D, g, blk = c["tokens"], c["num_kv_heads"], c["head_size"], c["group_size"], c["block_size"]
    T = tokens or T
    nb = T // blk
    k = torch.randn(T, H, D, device=device).to(torch.bfloat16)
    v = torch.randn(T, H, D, device=device).to(torch.bfloat16)
    slots = torch.randperm(nb, device=device).repeat_interleave(blk) * blk + torch.arange(T, device=device) % blk
    f = lambda *s, dt=torch.float32: torch.zeros(s, dtype=dt, device=device)
    views = (f(nb, H, D, blk // 8, dt=torch.int32), f(nb, H, D, blk // g), f(nb, H, D, blk // g),
             f(nb, blk, H, D // 8, dt=torch.int32), f(nb, blk, H, D // g), f(nb, blk, H, D // g))

    def once():  # the bulk prompt write's flush of both sides: one launch
        kivi_pack_kv_cache(k, v, slots, views[:3], views[3:], g, validate_slots=False)

    # the launch replayed from a CUDA graph (the device work alone, not
    # the Python wrappers' launch overhead); the inputs (33 MB) fit in L2, so
    # a 256 MB buffer is written before every timed replay
    t = time_loop_flushed(once, 20, 3, device) * 1e-3
    by = T * (H * D * 2 * 2 + H * (D // 2 + 8 * D // g) * 2)
    res = {"gbs": by / t / 1e9, "bytes_per_call": by, "us_per_call": t * 1e6, "tokens": T,
           "bytes_per_token": by // T, "launches_per_call": 1, "entry": "qkv_kivi_pack_kv"}
    if check:
        res.update(cpu_check_pack(k, v, slots, views, g, by))
    return res


def cpu_check_pack(k, v, slots, views, g, by, runs=5):
    """The reference's pack arithmetic (oracle/ numpy port of the
    layout-exact CPU packers) on the same inputs: bit-exact comparison of all
    six views, and its GB/s on the host (1 warm-up, median of ``runs``)."""
    import numpy as np

    O = _oracle()
    kn, vn = k.float().cpu().numpy(), v.float().cpu().numpy()
    sn = slots.cpu().numpy()
    ov = [np.zeros(x.shape, x.cpu().numpy().dtype) for x in views]

    def run():
        O.kivi_pack_key(kn, sn, ov[0], ov[1], ov[2], g)
        O.kivi_pack_value(vn, sn, ov[3], ov[4], ov[5], g)

    run()
    names = ("k_quant", "k_scale", "k_mn", "v_quant", "v_scale", "v_mn")
    exact = {n: bool(np.array_equal(x.cpu().numpy().view(np.uint32), o.view(np.uint32)))
             for n, x, o in zip(names, views, ov)}
    times = []
    for _ in range(runs):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    info = cpu_info()
    return {"parity": {"bit_exact": all(exact.values()), "views": exact, "tokens": int(kn.shape[0])},
            "cpu_baseline": {"value": by / t / 1e9, "unit": "GB/s", "cores": info["cores"], "kind": "port",
                             "sample": f"the same {kn.shape[0]} tokens (keys and values): 1 warm-up, median of "
                                       f"{runs} runs", "cpu_model": info["cpu_model"],
                             "torch_threads": info["torch_threads"]}}


def e2e_impl(w, device):
    """A KIVI mixin bound to the workload's buffers, with its window state
    set to what the reference's writes leave (rows b = request b)."""
    import torch

    from qkv_b200.methods.kivi_int4.attention_backend import AscendKiviInt4AttentionBackendMixin

    class Host:
        pass

    class Impl(AscendKiviInt4AttentionBackendMixin, Host):
        pass

    impl = Impl()
    impl.num_heads, impl.num_kv_heads, impl.head_size = w.Hql, w.Hl, w.D
    impl.num_queries_per_kv = w.Hql // w.Hl
    impl.scale = w.D ** -0.5
    impl._init_kivi_state("kivi_int4", SimpleNamespace(
        cache_config=SimpleNamespace(kivi_group_size=w.g, kivi_residual_length=w.r),
        scheduler_config=SimpleNamespace(max_num_seqs=w.B + 1)))
    impl._bind_kivi_cache((w.kbuf, w.vbuf))
    impl.kivi_residual_key_cache.copy_(w.rk)
    impl.kivi_residual_value_cache.copy_(w.rv)
    bt = w.bt.numpy()
    for b in range(w.B):
        row = impl._get_kivi_residual_row(f"req{b}", create=True)
        assert row == b
        for side in (impl._kivi_planner.key, impl._kivi_planner.value):
            for i in range(w.res):
                p = w.hist + i
                side.slots[row, i] = int(bt[b, p // w.blk]) * w.blk + p % w.blk
            side.start[row] = 0
            side.length[row] = w.res
    return impl


def run_e2e(w, device, steps, warmup, world=1, rank=0):
    """tokens/s/layer through the plugin API with host buffers in the loop:
    per step, pinned q/k/v of this rank's heads go in, the mixin's forward
    runs (window planning, packs, decode), N > 1 gathers every rank's heads
    with ``qkv_b200.distributed.gather_heads``, and the full output comes back
    to the host. As a serving engine does, the copies run on their own
    streams into double-buffered device slots: step i + 1's inputs go up while
    step i computes, and step i's output comes down while step i + 1 runs
    (issued after step i + 1 is enqueued, so it never holds up that step's
    own host-to-device copy); every step's copies are inside the timed
    region."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from qkv_b200.distributed import HeadShard, PeerGather, gather_heads

    impl = e2e_impl(w, device)
    B, Hq, H, D = w.B, w.Hql, w.Hl, w.D
    shard = HeadShard(rank, world, num_kv_heads=H * world, num_heads=Hq * world)
    peer = PeerGather(shard, B, D, device) if world > 1 else None
    bt_host = w.bt.numpy()
    total = steps + warmup
    gen = torch.Generator().manual_seed(7)
    q_h = torch.randn(total, B, Hq, D, generator=gen).to(torch.bfloat16).pin_memory()
    k_h = torch.randn(total, B, H, D, generator=gen).to(torch.bfloat16).pin_memory()
    v_h = torch.randn(total, B, H, D, generator=gen).to(torch.bfloat16).pin_memory()
    out_h = torch.empty(B, Hq * world, D, dtype=torch.bfloat16).pin_memory()
    bt_pinned = w.bt.clone().pin_memory()
    lens = [w.L] * B
    names = [f"req{b}" for b in range(B)]
    # the runner's host copy of each step's slot mapping (pinned), as it has
    # one for q / k / v: the plugin reads it without a device round trip
    pos = w.L + np.arange(total)[:, None]  # position of each step's new token
    slots_h = torch.from_numpy(bt_host[np.arange(B)[None, :], pos // w.blk].astype(np.int64) * w.blk
                               + pos % w.blk).pin_memory()
    q_lens = list(range(1, B + 1))
    compute = torch.cuda.current_stream(device)
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    q_d = torch.empty(2, B, Hq, D, dtype=torch.bfloat16, device=device)
    k_d = torch.empty(2, B, H, D, dtype=torch.bfloat16, device=device)
    v_d = torch.empty(2, B, H, D, dtype=torch.bfloat16, device=device)
    out_d = torch.empty(2, B, Hq, D, dtype=torch.bfloat16, device=device)
    res_d = torch.empty(2, B, Hq * world, D, dtype=torch.bfloat16, device=device) if world > 1 else None
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]  # slot's inputs consumed by the forward
    ev_out = [torch.cuda.Event() for _ in range(2)]
    ev_read = [torch.cuda.Event() for _ in range(2)]  # slot's output copied to the host
    res = [None, None]
    for e in ev_used + ev_read:
        e.record(compute)

    def upload(i):
        s = i & 1
        up.wait_event(ev_used[s])
        with torch.cuda.stream(up):
            q_d[s].copy_(q_h[i], non_blocking=True)
            k_d[s].copy_(k_h[i], non_blocking=True)
            v_d[s].copy_(v_h[i], non_blocking=True)
        ev_in[s].record(up)

    def step(i):
        s = i & 1
        for b in range(B):
            lens[b] += 1
        md = SimpleNamespace(
            attn_state=SimpleNamespace(name="DecodeOnly"), actual_seq_lengths_q=q_lens,
            seq_lens_list=list(lens), slot_mapping=slots_h[i], block_tables=bt_pinned, req_ids=names,
            num_actual_tokens=B, causal=True, finished_req_ids=None,
        )
        compute.wait_event(ev_in[s])
        compute.wait_event(ev_read[s])
        impl.forward(None, q_d[s], k_d[s], v_d[s], (w.kbuf, w.vbuf), md, out_d[s])
        ev_used[s].record(compute)
        if i + 1 < total:
            upload(i + 1)
        # the gathered heads leave the peer buffer at once (its next call
        # reuses it): into this step's slot, which the download reads
        res[s] = gather_heads(out_d[s], shard, out=None if res_d is None else res_d[s], peer=peer)
        ev_out[s].record(compute)
        # the previous step's output goes down now: queued behind this step's
        # host-to-device staging copy, not ahead of it
        if i > 0:
            download(i - 1)

    def download(i):
        s = i & 1
        down.wait_event(ev_out[s])
        with torch.cuda.stream(down):
            out_h.copy_(res[s], non_blocking=True)
        ev_read[s].record(down)

    upload(0)
    for i in range(warmup):
        step(i)
    download(warmup - 1)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for i in range(warmup, total):
        step(i)
    download(total - 1)
    torch.cuda.synchronize(device)
    dt = (time.perf_counter() - t0) / max(steps, 1)
    h2d = B * (Hq + 2 * H) * D * 2 + B * 8 + B * 5 * 4 + B * 4 + w.bt.numel() * 4
    d2h = B * Hq * world * D * 2
    return dt, h2d, d2h


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    from qkv_b200.ops import kivi_paged_decode

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    cfg = dict(CONFIG5)
    cfg3 = dict(CONFIG3)
    if args.batch:
        cfg["batch"] = cfg3["batch"] = args.batch
    if args.only == "int8":
        run_only_int8(cfg3, rank, world, device, args)
        return
    if args.only == "config4":
        print(json.dumps({"only": "config4", **run_config4_leg(device, args)}), flush=True)
        return
    if args.only == "pack":
        res = bench_pack(device, check=args.check)
        res["at_32768_tokens"] = {k: v for k, v in bench_pack(device, tokens=32768).items()
                                  if k in ("gbs", "us_per_call", "tokens", "bytes_per_call")}
        print(json.dumps({"only": "pack", **res}), flush=True)
        return
    if args.only == "small":
        print(json.dumps({"only": "small", **run_small_configs(device, args)}), flush=True)
        return
    if args.only == "fp8":
        res = run_fp8_leg(cfg3, rank, world, device, args)
        if rank == 0:
            print(json.dumps({"only": "fp8", **res}), flush=True)
        return
    if args.only == "kivi" and args.shard:
        w = build_workload(cfg, 0, args.shard, device)
    else:
        w = build_workload(cfg, rank, world, device)
    out = torch.empty(w.B, w.Hql, w.D, dtype=torch.bfloat16, device=device)
    peer = None
    if world > 1:
        from qkv_b200.distributed import HeadShard, PeerGather

        peer = PeerGather(HeadShard(rank, world, num_kv_heads=cfg["num_kv_heads"], num_heads=cfg["num_heads"]),
                          w.B, w.D, device)
        full = torch.empty(w.B, cfg["num_heads"], w.D, dtype=torch.bfloat16, device=device)

    def decode():
        kivi_paged_decode(w.q, w.views, w.rk, w.rv, w.bt_dev, w.seq_lens, w.state, w.g, w.D ** -0.5, out, w.L)

    def step():
        if peer is None:
            decode()
            return
        # the decode leaves its split partials; one kernel merges them and
        # sends every rank's heads into every rank's [B, Hq, D]
        parts = kivi_paged_decode(w.q, w.views, w.rk, w.rv, w.bt_dev, w.seq_lens, w.state, w.g, w.D ** -0.5, out,
                                  w.L, partials=True)
        peer.gather_partials(parts, out, out=full)

    if args.only == "kivi":
        decode_ms = time_loop(decode, args.steps, args.warmup, device)
        print(json.dumps({"only": "kivi", "batch": w.B, "kv_heads": w.Hl, "decode_ms": decode_ms,
                          "gbs": algorithmic_bytes(w) / (decode_ms * 1e-3) / 1e9}), flush=True)
        return
    # warm-up on a side stream (allocator, NCCL communicators, kernel
    # attributes), then one decode step (decode + combine [+ all-gather])
    # captured as a CUDA graph: the serving loop replays it, so the timed
    # region measures the device, not Python's launch rate
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(max(args.warmup, 3)):
            step()
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    step_graph, decode_graph = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(step_graph):
        step()
    with torch.cuda.graph(decode_graph):
        decode()
    for _ in range(3):
        step_graph.replay()
    torch.cuda.synchronize(device)
    # parity of sampled requests against the reference's CPU path (which is
    # also the timed CPU baseline), before the timed region
    parity = None
    if world == 1 and args.check:
        decode()
        torch.cuda.synchronize(device)
        wc = SimpleNamespace(views=w.views, rk=w.rk, rv=w.rv, bt=w.bt, state=w.state, lens=[w.L] * w.B, q=w.q,
                             g=w.g, blk=w.blk, D=w.D)
        parity = cpu_check_kivi(wc, out, [0, w.B // 2 + 3], time_runs=5)
    sampler = ClockSampler(local)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        # every rank's clock poller is live before the barrier, so the ranks
        # enter the timed region together (a late rank would otherwise show
        # up as all-gather wait time on the others)
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize(device)
        start.record()
        for _ in range(args.steps):
            step_graph.replay()
        end.record()
        torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    # the decode call alone (dominant kernel), for the roofline
    ks, ke = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    ks.record()
    for _ in range(args.steps):
        decode_graph.replay()
    ke.record()
    torch.cuda.synchronize(device)
    decode_ms = ks.elapsed_time(ke) / args.steps
    if peer is None:
        # on one GPU the step IS the decode call (same graph work): one
        # measurement for both, so the kernel time cannot exceed the step's
        decode_ms = ms
    # graphs holding NCCL work are released before the process group goes
    del step_graph, decode_graph
    t = torch.tensor([ms, decode_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, decode_ms = t.tolist()

    from qkv_b200.ops import _lib

    workspace_splits = _lib.load().qkv_kivi_paged_decode_workspace(w.B, w.Hql, w.Hl, w.D, w.g, w.blk, w.L)
    # the page-pipelined decode kernel (history splits + window CTAs in one
    # grid), then the combine kernel when the plan has several splits
    launches_per_step = 2 if workspace_splits > 0 else 1

    pack = None
    if rank == 0:
        pack = bench_pack(device, check=world == 1 and args.check)
        pack["at_32768_tokens"] = {k: v for k, v in bench_pack(device, tokens=32768).items()
                                   if k in ("gbs", "us_per_call", "tokens", "bytes_per_call")}
    int8 = None
    if not args.no_int8:
        int8 = run_int8_leg(cfg3, rank, world, device, args)
    fp8 = None
    if not args.no_int8:
        fp8 = run_fp8_leg(cfg3, rank, world, device, args)
    small = None
    if world == 1 and not args.no_config4:
        small = run_small_configs(device, args)
    config4 = None
    if world == 1 and not args.no_config4:
        config4 = run_config4_leg(device, args)
    e2e_dt, h2d, d2h = (None, 0, 0)
    if args.e2e_steps > 0:
        e2e_dt, h2d, d2h = run_e2e(w, device, min(args.e2e_steps, 246), 10, world, rank)
        t = torch.tensor([e2e_dt], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_dt = float(t.item())

    if rank == 0:
        peaks = measured_peaks()
        peak = peaks.get("hbm_gbs")
        peak_src = "measured" if peak else "fallback"
        peak = peak or 6650.0
        by = algorithmic_bytes(w)
        achieved = by / (decode_ms * 1e-3) / 1e9
        value = w.B / (ms * 1e-3)
        cpu = None
        if parity is not None and "cpu" in parity:
            c = parity.pop("cpu")
            cpu = {"value": c["value"], "unit": UNIT, "cores": c["cores"], "kind": "port",
                   "sample": f"{c['sample']} of the workload (64 q / 8 kv heads): 1 warm-up, median of "
                             f"{c['runs']} runs; the CPU path is linear in requests",
                   "seconds_per_request": c["seconds_per_request"], "cpu_model": c["cpu_model"],
                   "cpu_count": c["cpu_count"], "torch_threads": c["torch_threads"]}
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "int4/bf16->fp32",
            "data": "synthetic",
            "config": workload_config(cfg, world),
            "hbm_gbs": achieved,
            "hbm_frac_of_8tbs": achieved / 8000.0,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": profiled_traffic("kivi_decode_tma_config5.md", world),
                         "traffic_source": "profiles/kivi_decode_tma_config5.md (ncu, 1 GPU, scaled 1/N)",
                         "peak_source": peak_src,
                         "bytes_per_launch": by, "kernel_ms": decode_ms},
            "parity": parity,
            "pack": pack,
            "int8_config3": int8,
            "config4": config4,
            "fp8_decode": fp8,
            "config1": None if small is None else small["config1"],
            "config2": None if small is None else small["config2"],
            "e2e": None if e2e_dt is None else {
                "value": w.B / e2e_dt, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_dt * 1e3, "api": "AscendKiviInt4AttentionBackendMixin.forward (DecodeOnly)"},
            "cpu_baseline": cpu,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": sampler.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_int8_leg(cfg3, rank, world, device, args):
    """Config 3 (INT8, 64 x 8192): decode tokens/s/layer and HBM GB/s of the
    int8 paged decode on this rank's heads (max over ranks)."""
    import torch
    import torch.distributed as dist

    from qkv_b200.ops import int8_paged_decode

    w8 = build_int8_workload(cfg3, rank, world, device)
    out8 = torch.empty(w8.B, w8.Hql, w8.D, dtype=torch.bfloat16, device=device)

    def decode8():
        int8_paged_decode(w8.q, w8.kc, w8.vc, w8.k_aq, w8.v_aq, w8.bt_dev, w8.seq_lens, w8.D ** -0.5, out8, w8.L)

    parity = None
    if world == 1 and rank == 0 and args.check:
        decode8()
        torch.cuda.synchronize(device)
        parity = cpu_check_int8(w8, out8, [0, 37], time_runs=5)
    ms8 = time_loop(decode8, args.steps, args.warmup, device)
    t = torch.tensor([ms8], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms8 = float(t.item())
    peak = measured_peaks().get("hbm_gbs") or 6650.0
    by = int8_bytes(w8)
    gbs = by / (ms8 * 1e-3) / 1e9
    del w8, out8
    torch.cuda.empty_cache()
    return {"workload": "BASELINE config 3: INT8 decode, 64 x 8192, Hq 32 / KVH 8, head 128",
            "tokens_per_s_per_layer": cfg3["batch"] / (ms8 * 1e-3), "ms_per_step": ms8,
            "bytes_per_launch": by, "hbm_gbs": gbs, "frac_of_measured_hbm": gbs / peak,
            "frac_of_8tbs": gbs / 8000.0, "cpu_baseline": _leg_cpu(parity, "port"), "parity": parity}


def _leg_cpu(parity, kind):
    """The CPU-baseline entry of a leg: the timing its parity check made."""
    if not parity or "cpu" not in parity:
        return None
    c = parity.pop("cpu")
    return {"value": c["value"], "unit": c["unit"], "cores": c["cores"], "kind": kind,
            "sample": f"{c['sample']}: 1 warm-up, median of {c['runs']} runs", "cpu_model": c["cpu_model"],
            "torch_threads": c["torch_threads"]}


def run_fp8_leg(cfg3, rank, world, device, args):
    """FP8 per-token-head decode at config 3's shape (64 x 8192, Hq 32 / KVH
    8, head 128; the reference has no read path for this method, so no
    BASELINE config names it): K/V ~ N(0, 1) x a per-(token, head) magnitude
    e^U(-1, 1), stored by ``fp8_store`` through a permuted block table."""
    import torch
    import torch.distributed as dist

    from qkv_b200.ops import fp8_paged_decode, fp8_store

    B, L, Hq, H, D, blk = (cfg3[k] for k in ("batch", "context", "num_heads", "num_kv_heads", "head_size",
                                            "block_size"))
    Hl, Hql = H // world, Hq // world
    pages = L // blk
    nb = B * pages
    gen = torch.Generator(device=device).manual_seed(4322)
    cpu_gen = torch.Generator().manual_seed(4322)
    bt = torch.randperm(nb, generator=cpu_gen).view(B, pages).to(torch.int32)
    kd = torch.empty(nb, blk, Hl, D, dtype=torch.uint8, device=device)
    vd = torch.empty_like(kd)
    ks = torch.empty(nb, blk, Hl, 1, dtype=torch.float32, device=device)
    vs = torch.empty_like(ks)
    pos = torch.arange(L, device=device)
    for b in range(B):
        mag = torch.exp(torch.rand(L, Hl, 1, generator=gen, device=device) * 2 - 1)
        k = (torch.randn(L, Hl, D, generator=gen, device=device) * mag).to(torch.bfloat16)
        v = (torch.randn(L, Hl, D, generator=gen, device=device) * mag).to(torch.bfloat16)
        fp8_store(k, v, bt[b].to(device).long()[pos // blk] * blk + pos % blk, kd, ks, vd, vs)
    q = torch.randn(B, Hql, D, generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    bt_dev = bt.to(device)
    sl = torch.full((B,), L, dtype=torch.int32, device=device)

    def decode():
        fp8_paged_decode(q, kd, ks, vd, vs, bt_dev, sl, D ** -0.5, out, L)

    ms = time_loop(decode, args.steps, args.warmup, device)
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    peak = measured_peaks().get("hbm_gbs") or 6650.0
    # codes + one fp32 scale per (token, head) and side, q, out, block table
    by = B * (Hl * L * 2 * (D + 4) + 2 * Hql * D * 2 + 4 * pages)
    gbs = by / (ms * 1e-3) / 1e9
    del kd, vd, ks, vs
    torch.cuda.empty_cache()
    return {"workload": "FP8 per-token-head decode at config 3's shape: 64 x 8192, Hq 32 / KVH 8, head 128",
            "tokens_per_s_per_layer": B / (ms * 1e-3), "ms_per_step": ms, "bytes_per_launch": by,
            "hbm_gbs": gbs, "frac_of_measured_hbm": gbs / peak}


def run_only_int8(cfg3, rank, world, device, args):
    res = run_int8_leg(cfg3, rank, world, device, args)
    if rank == 0:
        print(json.dumps({"only": "int8", **res}), flush=True)


if __name__ == "__main__":
    main()
