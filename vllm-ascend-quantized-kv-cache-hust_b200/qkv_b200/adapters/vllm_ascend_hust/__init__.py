"""vllm-ascend-hust host: ``install_kv_impl_dispatch`` routes the quantized
cache dtypes of ``AscendAttentionBackend.get_impl_cls`` to this package."""

from .backend import install_kv_impl_dispatch

__all__ = ["install_kv_impl_dispatch"]
