"""Host adapters (vllm-ascend-hust)."""

from .base import HostAdapter

__all__ = ["HostAdapter"]
