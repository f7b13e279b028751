"""qkv_kivi_paged_decode_noalloc through the C ABI.

That entry point serves callers that cannot give this library a device
workspace (an engine whose KV-cache pool already owns the free device memory,
a host in another language without a device allocator, a serving loop that
must not call cudaMalloc): the split-KV partials live in a static device array
inside the library instead. Its output must equal the workspace entry point's
on the same inputs, bit for bit, call after call — the array keeps the previous call's
contents, so two calls in a row with different inputs check that nothing
stale leaks through. Collected last (file name), so a first-failure run has
already exercised every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from qkv_b200.ops import _lib, kivi_pack_key_cache, kivi_pack_value_cache
from qkv_b200.ops._torch import WORKSPACE

pytestmark = pytest.mark.gpu


def _case(seed, B, lens, Hq, H, D, g, blk, cap, dev):
    gen = torch.Generator(device=dev).manual_seed(seed)
    maxb = max((L + blk - 1) // blk for L in lens)
    nb = B * maxb + 1
    f = lambda *s, dt=torch.float32: torch.zeros(s, dtype=dt, device=dev)
    views = (f(nb, H, D, blk // 8, dt=torch.int32), f(nb, H, D, blk // g) + 1, f(nb, H, D, blk // g),
             f(nb, blk, H, D // 8, dt=torch.int32), f(nb, blk, H, D // g) + 1, f(nb, blk, H, D // g))
    bt = torch.randperm(nb - 1, device=dev)[: B * maxb].view(B, maxb).to(torch.int32)
    res_k = torch.randn(B, cap, H, D, generator=gen, device=dev).to(torch.bfloat16)
    res_v = torch.randn(B, cap, H, D, generator=gen, device=dev).to(torch.bfloat16)
    state = []
    for b, L in enumerate(lens):
        hist = ((L - 1) // g) * g  # whole key groups; the window keeps 1..g <= cap tokens
        pos = torch.arange(hist, device=dev)
        slots = bt[b].long()[pos // blk] * blk + pos % blk
        k = torch.randn(hist, H, D, generator=gen, device=dev).to(torch.bfloat16)
        v = torch.randn(hist, H, D, generator=gen, device=dev).to(torch.bfloat16)
        kivi_pack_key_cache(k, slots, *views[:3], g)
        kivi_pack_value_cache(v, slots, *views[3:], g)
        state.append([b, b % cap, L - hist, (3 * b) % cap, L - hist, L])
    q = torch.randn(B, Hq, D, generator=gen, device=dev).to(torch.bfloat16)
    return (q, views, res_k, res_v, bt, torch.tensor(lens, dtype=torch.int32, device=dev),
            torch.tensor(state, dtype=torch.int32, device=dev))


def _call(noalloc, q, views, res_k, res_v, bt, sl, st, Hq, H, D, g, blk, out):
    lib = _lib.load()
    B = q.shape[0]
    L = int(sl.max())
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    head = [p(q), q.stride(0), *(p(v) for v in views), p(res_k), p(res_v), res_k.shape[0], res_k.shape[1],
            p(bt), bt.stride(0), p(sl), p(st), B, Hq, H, D, g, blk, views[0].shape[0], L, D ** -0.5]
    if noalloc:
        rc = lib.qkv_kivi_paged_decode_noalloc(*head, p(out), out.stride(0), stream)
    else:
        need = lib.qkv_kivi_paged_decode_workspace(B, Hq, H, D, g, blk, L)
        ws = WORKSPACE.get(q.device, need)
        rc = lib.qkv_kivi_paged_decode(*head, None if ws is None else p(ws), 0 if ws is None else ws.numel(),
                                       p(out), out.stride(0), stream)
    _lib.check(rc, "noalloc" if noalloc else "workspace")


@pytest.mark.parametrize("group", [128, 64])
def test_noalloc_decode_matches_workspace_entry_point_twice(group):
    dev = torch.device("cuda", 0)
    Hq, H, D, blk, cap = 40, 8, 128, 128, 128
    for call, (seed, lens) in enumerate([(1, [3000, 8192, 1500, 129]), (2, [700, 4100, 6000])]):
        args = _case(seed + group, len(lens), lens, Hq, H, D, group, blk, cap, dev)
        want = torch.full((len(lens), Hq, D), float("nan"), dtype=torch.bfloat16, device=dev)
        got = torch.full_like(want, float("nan"))
        _call(False, *args, Hq, H, D, group, blk, want)
        _call(True, *args, Hq, H, D, group, blk, got)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all(), f"call {call}: unwritten outputs"
        # same split plan, same kernels, same inputs: bit for bit, so stale
        # scratch from the previous call cannot hide inside a tolerance
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), f"call {call}"
        code = _lib.device_error(torch.cuda.current_stream().cuda_stream)
        assert code == 0


def test_noalloc_rejects_batches_beyond_its_scratch():
    lib = _lib.load()
    B, Hq, H, D, g, blk, L = 512, 64, 8, 128, 128, 128, 1 << 17
    assert lib.qkv_kivi_paged_decode_workspace(B, Hq, H, D, g, blk, L) > 8 << 20
    dummy = ctypes.c_void_p(16)
    rc = lib.qkv_kivi_paged_decode_noalloc(
        dummy, Hq * D, *([dummy] * 8), 4, 128, dummy, 1024, dummy, dummy,
        B, Hq, H, D, g, blk, 100, L, 0.1, dummy, Hq * D, None,
    )
    assert rc == _lib.QKV_ERR_WORKSPACE
    assert "static" in _lib.last_error()
