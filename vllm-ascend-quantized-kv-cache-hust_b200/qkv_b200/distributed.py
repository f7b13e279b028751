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


def gather_heads(local_out: torch.Tensor, shard: HeadShard, group=None,
                 gathered: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gathers every rank's ``[B, Hq/N, D]`` attention output into
    ``[B, Hq, D]`` (rank-major head order, i.e. the model's head order).
    One collective; ``gathered``/``out`` may be preallocated."""
    import torch.distributed as dist

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


__all__ = ["HeadShard", "gather_heads"]
