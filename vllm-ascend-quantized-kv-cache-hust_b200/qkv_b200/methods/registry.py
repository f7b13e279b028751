"""Method registry (fail closed on unknown names), as methods/registry.py:21-66
of the reference."""

from __future__ import annotations

from typing import Any

from .base import KvQuantMethod, MethodConfig, MethodSpec

_REGISTRY: dict[str, MethodSpec] = {}


def register_method(spec: MethodSpec) -> MethodSpec:
    if spec.name in _REGISTRY:
        raise ValueError(f"method {spec.name!r} is already registered")
    _REGISTRY[spec.name] = spec
    return spec


def known_methods() -> tuple[str, ...]:
    return tuple(sorted(_REGISTRY))


def list_methods(host: str | None = None) -> tuple[str, ...]:
    if host is None:
        return known_methods()
    return tuple(n for n in known_methods() if host in _REGISTRY[n].supports)


def get_spec(name: str) -> MethodSpec:
    spec = _REGISTRY.get(name)
    if spec is None:
        known = ", ".join(known_methods()) or "<none>"
        raise ValueError(f"unknown quantized KV method {name!r}; known: {known}")
    return spec


def get_method(name: str, **config_overrides: Any) -> KvQuantMethod:
    spec = get_spec(name)
    return KvQuantMethod(spec, MethodConfig(**config_overrides))


def reset_registry() -> None:
    _REGISTRY.clear()


__all__ = ["get_method", "get_spec", "known_methods", "list_methods", "register_method", "reset_registry"]
