"""Shared adapter type (the reference's adapters/base.py:14-44): host imports
happen inside methods only, so adapters build anywhere and fail closed when
their host is missing."""

from __future__ import annotations

import importlib.util
from typing import Any


class HostAdapter:
    host: str = ""
    host_module: str = ""

    def __init__(self, method: Any) -> None:
        self.method = method

    @classmethod
    def available(cls) -> bool:
        try:
            return importlib.util.find_spec(cls.host_module) is not None
        except (ImportError, ValueError):
            return False

    def require_host(self) -> None:
        if not self.available():
            raise RuntimeError(
                f"host adapter {type(self).__name__} requires {self.host_module!r}, "
                "which is not importable in this environment"
            )

    def register(self, **options: Any) -> dict[str, Any]:
        raise NotImplementedError


__all__ = ["HostAdapter"]
