"""The decode's split partials merged by the fused combine + all-gather
kernel (qkv_kivi_paged_decode_partials + qkv_peer_combine_allgather) equal
the decode with its own combine, bit for bit. Run with one rank (world 1:
no peers, the kernel writes this rank's heads), so one GPU covers the merge
arithmetic; the multi-rank exchange is tests/test_gpu_peer_gather.py."""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_fused_combine_matches_decode_combine_on_one_rank():
    from qkv_b200.methods.kivi_int4.byte_cache import KiviByteCacheLayout, kivi_caches_from_byte_tensors
    from qkv_b200.ops import _lib, kivi_pack_key_cache, kivi_pack_value_cache, kivi_paged_decode
    from qkv_b200.ops._torch import stream_handle

    dev = torch.device("cuda", 0)
    B, Hq, H, D, g, blk, L = 6, 32, 8, 128, 128, 128, 5000
    gen = torch.Generator(device=dev).manual_seed(9)
    pages = (L + blk - 1) // blk
    nb = B * pages
    lay = KiviByteCacheLayout(num_blocks=nb, block_size=blk, num_kv_heads=H, head_size=D, group_size=g)
    kbuf = torch.zeros(nb, blk, H, lay.bytes_per_token_head, dtype=torch.uint8, device=dev)
    vbuf = torch.zeros_like(kbuf)
    views = kivi_caches_from_byte_tensors(kbuf, vbuf, lay)
    bt = torch.arange(nb, dtype=torch.int32, device=dev).view(B, pages)
    hist = (L // g) * g
    for b in range(B):
        k = torch.randn(hist, H, D, generator=gen, device=dev).to(torch.bfloat16)
        v = torch.randn(hist, H, D, generator=gen, device=dev).to(torch.bfloat16)
        slots = torch.arange(hist, device=dev) + b * pages * blk
        kivi_pack_key_cache(k, slots, *views[:3], g)
        kivi_pack_value_cache(v, slots, *views[3:], g)
    q = torch.randn(B, Hq, D, generator=gen, device=dev).to(torch.bfloat16)
    sl = torch.full((B,), hist, dtype=torch.int32, device=dev)
    want = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=dev)
    kivi_paged_decode(q, views, None, None, bt, sl, None, g, D ** -0.5, want, hist)

    lib = _lib.load()
    slice_bytes = B * Hq * D * 2
    buf = ctypes.c_void_p()
    _lib.check(lib.qkv_peer_alloc(slice_bytes, 1, ctypes.byref(buf)), "qkv_peer_alloc")
    try:
        buffers = (ctypes.c_void_p * 1)(buf.value)
        local = torch.empty_like(want)
        for _ in range(3):  # the epoch advances call to call
            parts = kivi_paged_decode(q, views, None, None, bt, sl, None, g, D ** -0.5, local, hist, partials=True)
            assert parts.splits > 1
            got = torch.full_like(want, float("nan"))
            rc = lib.qkv_peer_combine_allgather(
                parts.acc_ptr(), parts.ml_ptr(), parts.splits, B, Hq, D, local.data_ptr(),
                ctypes.addressof(buffers), slice_bytes, got.data_ptr(), 0, 1, stream_handle(dev))
            _lib.check(rc, "qkv_peer_combine_allgather")
            torch.cuda.synchronize(dev)
            assert torch.equal(got, want)
        code = _lib.device_error(torch.cuda.current_stream(dev).cuda_stream)
        assert code == 0, _lib.DEVICE_ERRORS.get(code, code)
    finally:
        torch.cuda.synchronize(dev)
        lib.qkv_peer_free(buf)
