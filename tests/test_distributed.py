"""KV-head sharding across ranks on CPU (gloo, world size 2).

Each rank keeps its KV heads and their query heads, computes attention for
them alone (here with the oracle's dense attention, the host-side stand-in
for the kernel), and one all-gather reassembles the output; it must equal
the single-rank result exactly. Also: shard geometry rules, and a rank that
never joins makes the others fail with a timeout instead of hanging.
"""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import qkv_oracle as O
from qkv_b200.distributed import HeadShard, gather_heads


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data():
    rng = np.random.default_rng(3)
    B, L, Hq, H, D = 3, 40, 8, 4, 16
    q = rng.standard_normal((B, Hq, D)).astype(np.float32)
    k = rng.standard_normal((B * L, H, D)).astype(np.float32)
    v = rng.standard_normal((B * L, H, D)).astype(np.float32)
    return q, k, v, B, L


def _worker(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        q, k, v, B, L = _data()
        shard = HeadShard(rank, world, num_kv_heads=k.shape[1], num_heads=q.shape[1])
        ql = shard.take_q(torch.from_numpy(q)).numpy()
        kl = shard.take_kv(torch.from_numpy(k)).numpy()
        vl = shard.take_kv(torch.from_numpy(v)).numpy()
        local = O.dense_attention(ql, kl, vl, [1] * B, [L] * B, 0.25, causal=True)
        full = gather_heads(torch.from_numpy(np.ascontiguousarray(local)), shard)
        if rank == 0:
            result.put(full.numpy())
    except Exception as exc:
        result.put(f"{type(exc).__name__}: {exc}")
        raise
    finally:
        dist.destroy_process_group()


def test_head_sharded_attention_equals_single_rank():
    world = 2
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    got = result.get(timeout=120)
    assert not isinstance(got, str), got
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k, v, B, L = _data()
    want = O.dense_attention(q, k, v, [1] * B, [L] * B, 0.25, causal=True)
    assert np.array_equal(got, want)


def _lonely(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
        t = torch.zeros(4)
        dist.all_reduce(t)
        result.put("completed")
    except Exception as exc:  # the missing peer must surface as an error
        result.put(type(exc).__name__)


def test_missing_rank_fails_with_timeout_not_hang():
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(0, 2, _free_port(), result))
    p.start()
    outcome = result.get(timeout=120)
    p.join(timeout=60)
    assert outcome != "completed"


def test_shard_geometry():
    s = HeadShard(1, 4, num_kv_heads=8, num_heads=64)
    assert s.kv_range == (2, 4) and s.q_range == (16, 32)
    assert s.local_kv_heads == 2 and s.local_heads == 16
    with pytest.raises(ValueError, match="divisible"):
        HeadShard(0, 3, num_kv_heads=8, num_heads=64)
    with pytest.raises(ValueError, match="bad rank"):
        HeadShard(4, 4, num_kv_heads=8, num_heads=64)
