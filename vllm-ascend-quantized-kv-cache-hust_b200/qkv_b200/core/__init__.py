"""Cross-cutting layer: host detection, activation, device guards (no heavy imports)."""

from .activation import activate
from .hosts import ALL_HOSTS, VLLM_ASCEND_HUST, detect_host, require_host_stack
from .runtime import cuda_sm100_available, require_cuda_sm100

__all__ = [
    "ALL_HOSTS",
    "VLLM_ASCEND_HUST",
    "activate",
    "cuda_sm100_available",
    "detect_host",
    "require_cuda_sm100",
    "require_host_stack",
]
