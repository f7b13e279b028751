"""FP8 per-token-head byte budget and the split of the host's two KV buffers.

The reference's contract (methods/fp8_per_token_head/byte_cache.py): the host
hands one layer two equal byte buffers; each is carved, in order, into two
views

    key buffer:   [k_data uint8 (NB, B, KVH, D) | k_scale f32 (NB, B, KVH, 1)]
    value buffer: [v_data uint8 (NB, B, KVH, D) | v_scale f32 (NB, B, KVH, 1)]

so a (token, head) costs ``S = D + 4`` bytes per side (E4M3 codes plus one
fp32 scale), the host's page budget ``2 * block * KVH * (D + 4)``. The data
bytes are E4M3 (``view(torch.float8_e4m3fn)``); ``D % 4 == 0`` keeps every
scale on a 4-byte boundary. The views alias the host memory.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from ...ops.kivi_layout import _check_contiguous


def _check_head_size(head_size: int) -> None:
    if head_size <= 0 or head_size % 4:
        raise ValueError(
            "fp8_per_token_head requires head_size positive and divisible "
            f"by 4, got {head_size}"
        )


@dataclass(frozen=True)
class Fp8PerTokenHeadLayout:
    """Shapes of one FP8 per-token-head paged allocation."""

    num_blocks: int
    block_size: int
    num_kv_heads: int
    head_size: int

    def __post_init__(self) -> None:
        if self.num_blocks <= 0:
            raise ValueError(f"num_blocks must be positive, got {self.num_blocks}")
        _check_head_size(self.head_size)

    def side_specs(self) -> tuple[tuple[tuple[int, ...], Any], ...]:
        nb, blk, kvh, d = self.num_blocks, self.block_size, self.num_kv_heads, self.head_size
        return (((nb, blk, kvh, d), torch.uint8), ((nb, blk, kvh, 1), torch.float32))

    key_specs = side_specs
    value_specs = side_specs

    @property
    def bytes_per_token_head(self) -> int:
        return self.head_size + 4

    @property
    def region_bytes(self) -> int:
        return self.num_blocks * self.block_size * self.num_kv_heads * self.bytes_per_token_head

    def page_size_bytes(self) -> int:
        """Bytes of one block across both sides (the host allocator's page)."""
        return 2 * self.block_size * self.num_kv_heads * self.bytes_per_token_head

    def compression_vs_fp16(self) -> float:
        return (2 * self.head_size) / self.bytes_per_token_head

    def describe(self) -> dict[str, Any]:
        return {
            "region_bytes": self.region_bytes,
            "bytes_per_token": 2 * self.num_kv_heads * self.bytes_per_token_head,
            "compression_vs_fp16": self.compression_vs_fp16(),
            "side": [{"shape": list(s), "dtype": str(t).replace("torch.", "")} for s, t in self.side_specs()],
        }


def fp8_per_token_head_layout(key_cache: torch.Tensor, value_cache: torch.Tensor, *, num_kv_heads: int,
                              head_size: int) -> Fp8PerTokenHeadLayout:
    """Derives the layout from the two host buffers (the block size is what
    the byte count leaves): ``region = NB * block * KVH * (D + 4)``."""
    _check_contiguous("key_cache", key_cache)
    _check_contiguous("value_cache", value_cache)
    if key_cache.device != value_cache.device:
        raise RuntimeError(
            f"fp8_per_token_head key/value caches must share a device, got {key_cache.device} and "
            f"{value_cache.device}."
        )
    kb = key_cache.numel() * key_cache.element_size()
    vb = value_cache.numel() * value_cache.element_size()
    if kb != vb:
        raise RuntimeError(
            f"fp8_per_token_head key cache holds {kb} bytes but value cache holds {vb}; the layout needs "
            "equal regions."
        )
    _check_head_size(head_size)
    nb = int(key_cache.shape[0])
    stride = nb * num_kv_heads * (head_size + 4)
    if stride <= 0 or kb % stride:
        raise RuntimeError(
            f"fp8_per_token_head cache region of {kb} bytes is not a whole number of pages for "
            f"head_size={head_size}, num_kv_heads={num_kv_heads}, num_blocks={nb}."
        )
    return Fp8PerTokenHeadLayout(num_blocks=nb, block_size=kb // stride, num_kv_heads=num_kv_heads,
                                 head_size=head_size)


def _carve(cache: torch.Tensor, specs, region_bytes: int, name: str) -> list[torch.Tensor]:
    if not cache.is_contiguous():
        raise RuntimeError(f"fp8_per_token_head {name} cache must be contiguous.")
    have = cache.numel() * cache.element_size()
    if have != region_bytes:
        raise RuntimeError(f"fp8_per_token_head {name} cache must hold {region_bytes} bytes, got {have}.")
    flat = cache.reshape(-1).view(torch.uint8)
    out, off = [], 0
    for shape, dtype in specs:
        n = 1
        for d in shape:
            n *= d
        n *= dtype.itemsize
        out.append(flat.narrow(0, off, n).view(dtype).view(shape))
        off += n
    return out


def fp8_caches_from_byte_tensors(key_cache: torch.Tensor, value_cache: torch.Tensor,
                                 layout: Fp8PerTokenHeadLayout) -> tuple[torch.Tensor, ...]:
    """(k_data, k_scale, v_data, v_scale) views aliasing the two buffers."""
    k = _carve(key_cache, layout.key_specs(), layout.region_bytes, "key")
    v = _carve(value_cache, layout.value_specs(), layout.region_bytes, "value")
    return (*k, *v)


__all__ = ["Fp8PerTokenHeadLayout", "fp8_caches_from_byte_tensors", "fp8_per_token_head_layout"]
