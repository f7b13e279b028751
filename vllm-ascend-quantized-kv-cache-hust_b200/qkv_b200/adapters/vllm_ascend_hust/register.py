"""Registers the quantized-KV implementations with the host
(the reference's adapters/vllm_ascend_hust/register.py:19-52): installs the
``get_impl_cls`` dispatcher; the cache dtype literal selects the impl at run
time."""

from __future__ import annotations

from typing import Any

from ..base import HostAdapter

_PACKAGE = "qkv_b200.adapters.vllm_ascend_hust.backend"

BACKEND_CLASS_PATH_BY_DTYPE = {
    "int8": f"{_PACKAGE}:AscendInt8KvAttentionBackend",
    "kivi_int4": f"{_PACKAGE}:AscendKiviInt4KvAttentionBackend",
}


class AscendHustAdapter(HostAdapter):
    host = "vllm_ascend_hust"
    host_module = "vllm_ascend"

    def register(self) -> dict[str, Any]:
        self.require_host()
        cache_dtype = self.method.spec.dtype
        backend_class_path = BACKEND_CLASS_PATH_BY_DTYPE.get(cache_dtype)
        if backend_class_path is None:
            raise ValueError(
                f"method {self.method.name!r} has dtype {cache_dtype!r}, which the "
                "vllm-ascend-hust adapter cannot select; known dtypes: "
                f"{', '.join(sorted(BACKEND_CLASS_PATH_BY_DTYPE))}"
            )
        from .backend import install_kv_impl_dispatch

        host_backend = install_kv_impl_dispatch()
        return {
            "host": self.host,
            "method": self.method.name,
            "attention_backend": f"{host_backend.__module__}.{host_backend.__name__}",
            "backend_class_path": backend_class_path,
            "integration": "host_get_impl_cls_dispatch",
            "cache_dtype_literal": cache_dtype,
            "usage": f"vllm serve MODEL --kv-cache-dtype {cache_dtype}",
        }


__all__ = ["AscendHustAdapter", "BACKEND_CLASS_PATH_BY_DTYPE"]
