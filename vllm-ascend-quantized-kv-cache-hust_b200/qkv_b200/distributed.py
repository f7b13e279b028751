"""KV-head sharding of the quantized-KV attention path across GPUs.

Attention, the INT8 scales and the KIVI pack are independent per KV head, so
the path shards like vLLM tensor parallelism: rank i of N owns KV heads
``[H*i/N, H*(i+1)/N)`` and the query heads that read them, keeps its heads'
share of both cache buffers (the same ``KiviByteCacheLayout`` with
``num_kv_heads = H/N``, so the byte budget per head is unchanged) and of the
residual windows, and computes its heads' attention with no exchange. One
all-gather of the ``[B, Hq/N, D]`` outputs reassembles ``[B, Hq, D]``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    num_kv_heads: int   # of the whole model
    num_heads: int      # query heads of the whole model

    def __post_init__(self) -> None:
        if self.world <= 0 or not 0 <= self.rank < self.world:
            raise ValueError(f"bad rank {self.rank} of {self.world}")
        if self.num_kv_heads % self.world:
            raise ValueError(
                f"num_kv_heads ({self.num_kv_heads}) must be divisible by the world size ({self.world})"
            )
        if self.num_heads % self.num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")

    @property
    def local_kv_heads(self) -> int:
        return self.num_kv_heads // self.world

    @property
    def local_heads(self) -> int:
        return self.num_heads // self.world

    @property
    def kv_range(self) -> tuple[int, int]:
        n = self.local_kv_heads
        return self.rank * n, (self.rank + 1) * n

    @property
    def q_range(self) -> tuple[int, int]:
        n = self.local_heads
        return self.rank * n, (self.rank + 1) * n

    def take_kv(self, x: torch.Tensor, dim: int = -2) -> torch.Tensor:
        """This rank's KV heads of a ``[..., KVH, D]`` tensor."""
        a, b = self.kv_range
        return x.narrow(dim, a, b - a)

    def take_q(self, x: torch.Tensor, dim: int = -2) -> torch.Tensor:
        """This rank's query heads of a ``[..., Hq, D]`` tensor."""
        a, b = self.q_range
        return x.narrow(dim, a, b - a)


class PeerGather:
    """All-gather of the sharded ``[B, Hq/N, D]`` outputs over NVLink peer
    memory (``qkv_peer_allgather``): one kernel per call sends this rank's
    heads into every peer's receive buffer, each word stored together with
    the call's epoch, and assembles ``[B, Hq, D]`` from what the peers sent
    (no barrier; graph-capturable; waits bounded). Built collectively: every
    rank constructs it with the same arguments (its buffer's CUDA IPC handle
    goes to the others through ``all_gather_object``) and makes the same
    ``gather`` calls in order."""

    def __init__(self, shard: HeadShard, max_batch: int, head_size: int, device: torch.device | str,
                 group=None) -> None:
        import ctypes

        import torch.distributed as dist

        from .ops import _lib

        if shard.world > 8:
            raise ValueError("PeerGather supports up to 8 ranks")
        self._lib = lib = _lib.load()
        self.shard, self.device, self.group = shard, torch.device(device), group
        self.max_batch, self.head_size = max_batch, head_size
        self.row_bytes = shard.local_heads * head_size * 2
        self.slice_bytes = (max_batch * self.row_bytes + 15) // 16 * 16
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(lib.qkv_peer_alloc(self.slice_bytes, shard.world, ctypes.byref(own)), "qkv_peer_alloc")
            handle = ctypes.create_string_buffer(64)
            _lib.check(lib.qkv_ipc_handle(own, handle), "qkv_ipc_handle")
            handles: list = [None] * shard.world
            dist.all_gather_object(handles, handle.raw, group=group)
            peers = []
            for r, h in enumerate(handles):
                if r == shard.rank:
                    peers.append(own.value)
                    continue
                p = ctypes.c_void_p()
                _lib.check(lib.qkv_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p)), "qkv_ipc_open")
                peers.append(p.value)
        self._own, self._peers = own.value, peers
        self._buffers = (ctypes.c_void_p * shard.world)(*peers)
        self._buffers_ptr = ctypes.addressof(self._buffers)

    def gather(self, local_out: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """``local_out`` bf16 ``[B, Hq/N, D]`` contiguous -> ``out`` (or a new
        tensor) bf16 ``[B, Hq, D]``."""
        from .ops import _lib
        from .ops._torch import require_cuda, stream_handle

        B = local_out.shape[0]
        if (local_out.dtype != torch.bfloat16 or not local_out.is_contiguous() or B > self.max_batch
                or tuple(local_out.shape[1:]) != (self.shard.local_heads, self.head_size)):
            raise RuntimeError(f"PeerGather: expected contiguous bf16 [<= {self.max_batch}, "
                               f"{self.shard.local_heads}, {self.head_size}]")
        if out is None:
            out = torch.empty(B, self.shard.num_heads, self.head_size, dtype=torch.bfloat16, device=self.device)
        elif (out.dtype != torch.bfloat16 or not out.is_contiguous()
              or tuple(out.shape) != (B, self.shard.num_heads, self.head_size)):
            raise RuntimeError("PeerGather: out must be contiguous bf16 [B, Hq, D]")
        require_cuda("PeerGather", local_out, out)
        rc = self._lib.qkv_peer_allgather(local_out.data_ptr(), B, self.row_bytes, self._buffers_ptr,
                                          self.slice_bytes, out.data_ptr(), self.shard.rank, self.shard.world,
                                          stream_handle(self.device))
        _lib.check(rc, "qkv_peer_allgather")
        return out

    def gather_partials(self, partials, local_out: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """The split combine of a decode fused with the gather
        (``qkv_peer_combine_allgather``): ``partials`` is the
        ``DecodePartials`` that ``kivi_paged_decode(..., partials=True)``
        returned for ``local_out`` bf16 ``[B, Hq/N, D]``; -> ``out`` (or a
        new tensor) bf16 ``[B, Hq, D]``."""
        from .ops import _lib
        from .ops._torch import require_cuda, stream_handle

        if partials.splits <= 1:
            return self.gather(local_out, out=out)
        B = partials.batch
        if (partials.num_heads != self.shard.local_heads or partials.head_size != self.head_size
                or B > self.max_batch or local_out.shape[0] != B):
            raise RuntimeError("PeerGather: partials of another geometry")
        if out is None:
            out = torch.empty(B, self.shard.num_heads, self.head_size, dtype=torch.bfloat16, device=self.device)
        elif (out.dtype != torch.bfloat16 or not out.is_contiguous()
              or tuple(out.shape) != (B, self.shard.num_heads, self.head_size)):
            raise RuntimeError("PeerGather: out must be contiguous bf16 [B, Hq, D]")
        require_cuda("PeerGather", partials.workspace, out)
        rc = self._lib.qkv_peer_combine_allgather(
            partials.acc_ptr(), partials.ml_ptr(), partials.splits, B, self.shard.local_heads, self.head_size,
            local_out.data_ptr(), self._buffers_ptr, self.slice_bytes, out.data_ptr(), self.shard.rank,
            self.shard.world, stream_handle(self.device))
        _lib.check(rc, "qkv_peer_combine_allgather")
        return out

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's. Collective: every
        rank of the group calls it. This rank's stream is synchronised and the
        ranks pass a barrier first, so no peer can still be running a call
        that stores into the buffer freed here."""
        if self._own is None:
            return
        import torch.distributed as dist

        torch.cuda.synchronize(self.device)
        if dist.is_initialized() and self.shard.world > 1:
            dist.barrier(group=self.group)
            torch.cuda.synchronize(self.device)
        for r, p in enumerate(self._peers):
            if r != self.shard.rank:
                self._lib.qkv_ipc_close(p)
        self._lib.qkv_peer_free(self._own)
        self._own = None


def gather_heads(local_out: torch.Tensor, shard: HeadShard, group=None,
                 gathered: torch.Tensor | None = None, out: torch.Tensor | None = None,
                 peer: PeerGather | None = None) -> torch.Tensor:
    """All-gathers every rank's ``[B, Hq/N, D]`` attention output into
    ``[B, Hq, D]`` (rank-major head order, i.e. the model's head order).
    With ``peer`` the NVLink peer all-gather runs (one kernel, writing the
    final layout); otherwise one NCCL collective and a head permute;
    ``gathered``/``out`` may be preallocated."""
    import torch.distributed as dist

    if shard.world > 1 and peer is not None:
        return peer.gather(local_out.contiguous(), out=out)
    if shard.world == 1:
        if out is not None:
            out.copy_(local_out)
            return out
        return local_out
    B, hl, D = local_out.shape
    if gathered is None:
        gathered = torch.empty((shard.world * B, hl, D), dtype=local_out.dtype, device=local_out.device)
    # rank-major [world * B, Hq/N, D] (the form every backend accepts)
    dist.all_gather_into_tensor(gathered, local_out.contiguous(), group=group)
    if out is None:
        out = torch.empty((B, shard.world * hl, D), dtype=local_out.dtype, device=local_out.device)
    out.view(B, shard.world, hl, D).copy_(gathered.view(shard.world, B, hl, D).permute(1, 0, 2, 3))
    return out


__all__ = ["HeadShard", "PeerGather", "gather_heads"]
