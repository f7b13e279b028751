"""KIVI INT4 byte budget and the six-view split of the host's two KV buffers.

The host (vLLM) hands one attention layer exactly two cache tensors. KIVI
writes six named arrays; both sides need the same number of bytes, so each
host buffer is carved, in order and without interleaving, into three views
(the reference's contract, methods/kivi_int4/byte_cache.py:32-223):

    key buffer:   [k_quant int32 (NB, KVH, D, B/8) | k_scale f32 (NB, KVH, D, B/g) | k_mn f32 (same)]
    value buffer: [v_quant int32 (NB, B, KVH, D/8) | v_scale f32 (NB, B, KVH, D/g) | v_mn f32 (same)]

Bytes per token, per head, per side: ``S = D/2 + 8*D/g`` (half a byte per int4
lane, plus one fp32 scale and one fp32 min per group amortised over the group).
The views alias the host memory: the kernels write the host's buffers.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from ...ops.kivi_layout import _check_contiguous
from .geometry import validate_kivi_geometry

_LANES_PER_WORD = 8


def _numel(shape: tuple[int, ...]) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


def _span(specs) -> int:
    return sum(_numel(shape) * dtype.itemsize for shape, dtype in specs)


@dataclass(frozen=True)
class KiviByteCacheLayout:
    """Shapes of one KIVI paged allocation and the split of its two buffers."""

    num_blocks: int
    block_size: int
    num_kv_heads: int
    head_size: int
    group_size: int

    def __post_init__(self) -> None:
        if self.num_blocks <= 0:
            raise ValueError(f"num_blocks must be positive, got {self.num_blocks}")
        validate_kivi_geometry(
            head_size=self.head_size,
            group_size=self.group_size,
            residual_length=self.group_size,
            block_size=self.block_size,
        )

    def key_specs(self):
        nb, h, d, b, g = self.num_blocks, self.num_kv_heads, self.head_size, self.block_size, self.group_size
        return (
            ((nb, h, d, b // _LANES_PER_WORD), torch.int32),
            ((nb, h, d, b // g), torch.float32),
            ((nb, h, d, b // g), torch.float32),
        )

    def value_specs(self):
        nb, h, d, b, g = self.num_blocks, self.num_kv_heads, self.head_size, self.block_size, self.group_size
        return (
            ((nb, b, h, d // _LANES_PER_WORD), torch.int32),
            ((nb, b, h, d // g), torch.float32),
            ((nb, b, h, d // g), torch.float32),
        )

    @property
    def key_bytes(self) -> int:
        return _span(self.key_specs())

    @property
    def value_bytes(self) -> int:
        return _span(self.value_specs())

    @property
    def region_bytes(self) -> int:
        if self.key_bytes != self.value_bytes:
            raise RuntimeError(
                "KIVI byte layout requires equal key/value regions, got "
                f"{self.key_bytes} vs {self.value_bytes}."
            )
        return self.key_bytes

    @property
    def bytes_per_token_head(self) -> int:
        return self.head_size // 2 + 8 * self.head_size // self.group_size

    @property
    def bytes_per_token(self) -> int:
        return 2 * self.num_kv_heads * self.bytes_per_token_head

    def compression_vs_fp16(self) -> float:
        return (2 * self.num_kv_heads * self.head_size * 2) / self.bytes_per_token

    def page_size_bytes(self) -> int:
        """Bytes of one block across both sides: what the host allocator needs
        (host shape ``(2, NB, block, KVH, S)`` uint8)."""
        return 2 * self.block_size * self.num_kv_heads * self.bytes_per_token_head

    def describe(self) -> dict[str, Any]:
        def summary(specs):
            return [{"shape": list(s), "dtype": str(t).replace("torch.", "")} for s, t in specs]

        return {
            "region_bytes": self.region_bytes,
            "bytes_per_token": self.bytes_per_token,
            "compression_vs_fp16": self.compression_vs_fp16(),
            "key": summary(self.key_specs()),
            "value": summary(self.value_specs()),
        }


def kivi_byte_cache_layout(key_cache: torch.Tensor, value_cache: torch.Tensor, *, num_kv_heads: int,
                           head_size: int, group_size: int) -> KiviByteCacheLayout:
    """Infers the paged layout from the two host buffers; the block size is
    ``bytes / (num_blocks * num_kv_heads * S)`` and must divide exactly."""
    _check_contiguous("key_cache", key_cache)
    _check_contiguous("value_cache", value_cache)
    if key_cache.device != value_cache.device:
        raise RuntimeError(
            f"KIVI key/value caches must share a device, got {key_cache.device} and {value_cache.device}."
        )
    kb = key_cache.numel() * key_cache.element_size()
    vb = value_cache.numel() * value_cache.element_size()
    if kb != vb:
        raise RuntimeError(
            f"KIVI key cache holds {kb} bytes but value cache holds {vb}; the int4 layout needs equal regions."
        )
    nb = int(key_cache.shape[0])
    s = head_size // 2 + 8 * head_size // group_size
    stride = nb * num_kv_heads * s
    if stride <= 0 or kb % stride:
        raise RuntimeError(
            f"KIVI cache region of {kb} bytes is not a whole number of pages for "
            f"head_size={head_size}, group_size={group_size}, num_kv_heads={num_kv_heads}, num_blocks={nb}."
        )
    return KiviByteCacheLayout(
        num_blocks=nb, block_size=kb // stride, num_kv_heads=num_kv_heads, head_size=head_size, group_size=group_size
    )


def _views(cache: torch.Tensor, specs, region_bytes: int, name: str) -> list[torch.Tensor]:
    if not cache.is_contiguous():
        raise RuntimeError(f"KIVI {name} cache must be contiguous.")
    have = cache.numel() * cache.element_size()
    if have != region_bytes:
        raise RuntimeError(f"KIVI {name} cache must hold {region_bytes} bytes, got {have}.")
    flat = cache.reshape(-1).view(torch.uint8)
    out, off = [], 0
    for shape, dtype in specs:
        n = _numel(shape) * dtype.itemsize
        out.append(flat.narrow(0, off, n).view(dtype).view(shape))
        off += n
    if off != flat.numel():
        raise RuntimeError(f"KIVI {name} region bookkeeping error: {off} vs {flat.numel()} bytes.")
    return out


def kivi_caches_from_byte_tensors(key_cache: torch.Tensor, value_cache: torch.Tensor,
                                  layout: KiviByteCacheLayout) -> tuple[torch.Tensor, ...]:
    """Two host buffers -> ``(k_quant, k_scale, k_mn, v_quant, v_scale, v_mn)``."""
    rb = layout.region_bytes
    return (*_views(key_cache, layout.key_specs(), rb, "key"), *_views(value_cache, layout.value_specs(), rb, "value"))


__all__ = ["KiviByteCacheLayout", "kivi_byte_cache_layout", "kivi_caches_from_byte_tensors"]
