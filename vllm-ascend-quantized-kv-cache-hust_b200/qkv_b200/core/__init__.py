"""Device guards of the kernel layer (no heavy imports)."""

from .runtime import cuda_sm100_available, require_cuda_sm100

__all__ = ["cuda_sm100_available", "require_cuda_sm100"]
