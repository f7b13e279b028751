"""NVLink peer all-gather of the KV-head-sharded outputs (qkv_peer_allgather)
against the expected head layout and against the NCCL all-gather, on 2 GPUs
as 2 processes (one per GPU). Skipped with fewer than 2 GPUs."""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, B: int, Hq: int, D: int) -> None:
    import datetime

    import torch.distributed as dist

    from qkv_b200.distributed import HeadShard, PeerGather, gather_heads
    from qkv_b200.ops import _lib

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        shard = HeadShard(rank, world, num_kv_heads=8, num_heads=Hq)
        hl = shard.local_heads
        peer = PeerGather(shard, B, D, dev)

        def local(step: int, b: int) -> torch.Tensor:
            # values that name (step, rank, request, head, dim)
            base = torch.arange(b * hl * D, device=dev, dtype=torch.float32).view(b, hl, D)
            return ((base + 1000.0 * rank + 7.0 * step) % 251.0).to(torch.bfloat16)

        def expected(step: int, b: int) -> torch.Tensor:
            base = torch.arange(b * hl * D, device=dev, dtype=torch.float32).view(b, hl, D)
            parts = [((base + 1000.0 * r + 7.0 * step) % 251.0).to(torch.bfloat16) for r in range(world)]
            return torch.cat(parts, dim=1)

        for step in range(20):
            b = B if step % 3 else B - 5  # ragged batches too
            x = local(step, b)
            got = peer.gather(x).clone()
            want = expected(step, b)
            assert torch.equal(got, want), f"rank {rank} step {step}"
            assert torch.equal(got, gather_heads(x, shard)), f"rank {rank} step {step} vs NCCL"
        # captured in a CUDA graph and replayed with new inputs
        x = local(100, B)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            peer.gather(x)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            res = peer.gather(x)
        for step in range(101, 106):
            x.copy_(local(step, B))
            g.replay()
            torch.cuda.synchronize(dev)
            assert torch.equal(res, expected(step, B)), f"rank {rank} graph step {step}"
        del g
        code = _lib.device_error(torch.cuda.current_stream(dev).cuda_stream)
        assert code == 0, _lib.DEVICE_ERRORS.get(code, code)
        dist.barrier()
        peer.close()
    finally:
        dist.destroy_process_group()


def _combine_worker(rank: int, world: int, port: int) -> None:
    """decode(partials) + qkv_peer_combine_allgather == decode + NCCL gather,
    bit for bit, on a KIVI cache sharded by KV head."""
    import datetime

    import torch.distributed as dist

    from qkv_b200.distributed import HeadShard, PeerGather, gather_heads
    from qkv_b200.methods.kivi_int4.byte_cache import KiviByteCacheLayout, kivi_caches_from_byte_tensors
    from qkv_b200.ops import kivi_pack_key_cache, kivi_pack_value_cache, kivi_paged_decode

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        B, Hq, KVH, D, g, blk, L = 8, 32, 8, 128, 128, 128, 6000
        shard = HeadShard(rank, world, num_kv_heads=KVH, num_heads=Hq)
        H, hl = shard.local_kv_heads, shard.local_heads
        gen = torch.Generator(device=dev).manual_seed(5)  # same full tensors on every rank
        pages = (L + blk - 1) // blk
        nb = B * pages
        lay = KiviByteCacheLayout(num_blocks=nb, block_size=blk, num_kv_heads=H, head_size=D, group_size=g)
        kbuf = torch.zeros(nb, blk, H, lay.bytes_per_token_head, dtype=torch.uint8, device=dev)
        vbuf = torch.zeros_like(kbuf)
        views = kivi_caches_from_byte_tensors(kbuf, vbuf, lay)
        bt = torch.arange(nb, dtype=torch.int32, device=dev).view(B, pages)
        hist = (L // 128) * 128
        for b in range(B):
            k = torch.randn(hist, KVH, D, generator=gen, device=dev).to(torch.bfloat16)
            v = torch.randn(hist, KVH, D, generator=gen, device=dev).to(torch.bfloat16)
            slots = torch.arange(hist, device=dev) + b * pages * blk
            kivi_pack_key_cache(shard.take_kv(k).contiguous(), slots, *views[:3], g)
            kivi_pack_value_cache(shard.take_kv(v).contiguous(), slots, *views[3:], g)
        q = shard.take_q(torch.randn(B, Hq, D, generator=gen, device=dev).to(torch.bfloat16)).contiguous()
        sl = torch.full((B,), hist, dtype=torch.int32, device=dev)
        out_a = torch.empty(B, hl, D, dtype=torch.bfloat16, device=dev)
        out_b = torch.empty_like(out_a)
        kivi_paged_decode(q, views, None, None, bt, sl, None, g, D ** -0.5, out_a, hist)
        want = gather_heads(out_a, shard)
        peer = PeerGather(shard, B, D, dev)
        for _ in range(3):
            parts = kivi_paged_decode(q, views, None, None, bt, sl, None, g, D ** -0.5, out_b, hist, partials=True)
            assert parts.splits > 1
            got = peer.gather_partials(parts, out_b)
            assert torch.equal(got, want), f"rank {rank}"
        dist.barrier()
        peer.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_combine_allgather_matches_decode_then_nccl():
    import torch.multiprocessing as mp

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_combine_worker, args=(2, _free_port()), nprocs=2, join=True)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("Hq", [64, 32])
def test_peer_allgather_matches_expected_and_nccl(Hq):
    import torch.multiprocessing as mp

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_worker, args=(2, _free_port(), 32, Hq, 128), nprocs=2, join=True)
