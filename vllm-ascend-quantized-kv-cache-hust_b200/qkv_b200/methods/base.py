"""Method model: descriptors, shared geometry config and the method handle.

The reference's zero-dependency method layer (methods/base.py:22-181): building
or registering a spec never imports torch, vllm or any device module.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping
from dataclasses import dataclass, field, replace
from typing import Any

from ..core.hosts import ALL_HOSTS
from ..dtypes import KVCacheLayout, KVQuantMode, resolve_layout


@dataclass(frozen=True)
class MethodConfig:
    """Geometry shared by every method; defaults as the reference
    (head 128, kv heads 8, q heads 32, block 128, group 128, residual 128)."""

    head_size: int = 128
    num_kv_heads: int = 8
    num_heads: int = 32
    block_size: int = 128
    group_size: int = 128
    residual_length: int = 128

    def validated(self) -> MethodConfig:
        if self.head_size <= 0:
            raise ValueError(f"head_size must be positive, got {self.head_size}")
        if self.num_kv_heads <= 0:
            raise ValueError(f"num_kv_heads must be positive, got {self.num_kv_heads}")
        if self.num_heads < self.num_kv_heads:
            raise ValueError(
                f"num_heads must be >= num_kv_heads, got {self.num_heads} < {self.num_kv_heads}"
            )
        if self.block_size <= 0:
            raise ValueError(f"block_size must be positive, got {self.block_size}")
        if self.group_size <= 0:
            raise ValueError(f"group_size must be positive, got {self.group_size}")
        if self.residual_length < 0:
            raise ValueError(f"residual_length must be non-negative, got {self.residual_length}")
        return self


@dataclass(frozen=True)
class MethodSpec:
    """Static description of one quantisation method (metadata only)."""

    name: str
    dtype: str
    summary: str
    quant_mode: KVQuantMode
    supports: tuple[str, ...]
    config_validator: Callable[[MethodConfig], None] | None = None
    adapter_factories: Mapping[str, Callable[[Any], Any]] = field(default_factory=dict)
    kernels: str = "libqkv_sm100 (sm_100a)"

    def describe(self) -> dict[str, Any]:
        return {
            "name": self.name,
            "dtype": self.dtype,
            "quant_mode": int(self.quant_mode),
            "summary": self.summary,
            "kernels": self.kernels,
            "supports": list(self.supports),
        }


class KvQuantMethod:
    """Method handle returned by ``registry.get_method``: layout contract,
    configuration and host adapter of one method."""

    def __init__(self, spec: MethodSpec, config: MethodConfig) -> None:
        if spec.config_validator is not None:
            spec.config_validator(config)
        self.spec = spec
        self.config = config.validated()

    @property
    def name(self) -> str:
        return self.spec.name

    @property
    def descriptor(self) -> dict[str, Any]:
        payload = self.spec.describe()
        payload["config"] = {
            f: getattr(self.config, f)
            for f in ("head_size", "num_kv_heads", "num_heads", "block_size", "group_size", "residual_length")
        }
        return payload

    def supports(self, host: str) -> bool:
        return host in self.spec.supports

    def resolve_layout(self) -> KVCacheLayout:
        return resolve_layout(self.spec.dtype, self.config.head_size)

    def host_adapter(self, host: str) -> Any:
        if host not in ALL_HOSTS:
            raise ValueError(f"unknown host {host!r}; known hosts: {', '.join(ALL_HOSTS)}")
        if not self.supports(host):
            raise ValueError(
                f"method {self.spec.name!r} does not support host {host!r} "
                f"(supports: {', '.join(self.spec.supports) or 'none'})"
            )
        factory = self.spec.adapter_factories.get(host)
        if factory is None:
            raise ValueError(f"method {self.spec.name!r} has no adapter wired for host {host!r} yet")
        return factory(self)

    def with_config(self, **overrides: Any) -> KvQuantMethod:
        return KvQuantMethod(self.spec, replace(self.config, **overrides))


__all__ = ["KvQuantMethod", "MethodConfig", "MethodSpec"]
