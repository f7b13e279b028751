"""Activation pipeline: method name -> host adapter -> register().

The reference's single activation path (core/activation.py:17-38), shared by
``kv_methods.activate`` and ``bootstrap.register_plugins``; unknown names,
bad configs, unknown hosts and missing host stacks all fail closed.
"""

from __future__ import annotations

from typing import Any


def activate(name: str, *, host: str | None = None, **config: Any) -> dict[str, Any]:
    from ..methods.registry import get_method
    from .hosts import ALL_HOSTS, require_host_stack

    if host is None:
        host = require_host_stack(f"activating method {name!r}")
    elif host not in ALL_HOSTS:
        raise ValueError(f"unknown host {host!r}; known hosts: {', '.join(ALL_HOSTS)}")
    method = get_method(name, **config)
    adapter = method.host_adapter(host)
    info = dict(adapter.register())
    info.setdefault("host", host)
    info["method"] = name
    return info


__all__ = ["activate"]
