"""vllm-ascend-hust host adapter."""

from .register import BACKEND_CLASS_PATH_BY_DTYPE, AscendHustAdapter

__all__ = ["AscendHustAdapter", "BACKEND_CLASS_PATH_BY_DTYPE"]
