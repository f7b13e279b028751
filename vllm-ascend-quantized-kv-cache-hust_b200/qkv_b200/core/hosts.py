"""Host detection: which serving stack this process runs in.

Same contract as the reference's core/hosts.py:28-46: the only host is
vllm-ascend-hust, detected by the importability of ``vllm_ascend`` (metadata
only, nothing is imported).
"""

from __future__ import annotations

import importlib.util

VLLM_ASCEND_HUST = "vllm_ascend_hust"
ALL_HOSTS = (VLLM_ASCEND_HUST,)


def _importable(name: str) -> bool:
    try:
        return importlib.util.find_spec(name) is not None
    except (ImportError, ValueError):
        return False


def detect_host() -> str | None:
    return VLLM_ASCEND_HUST if _importable("vllm_ascend") else None


def require_host_stack(what: str) -> str:
    host = detect_host()
    if host is None:
        raise RuntimeError(
            f"{what} requests quantized KV attention, but vllm_ascend is not "
            "importable; install the vllm-ascend-hust host stack first"
        )
    return host


__all__ = ["ALL_HOSTS", "VLLM_ASCEND_HUST", "detect_host", "require_host_stack"]
