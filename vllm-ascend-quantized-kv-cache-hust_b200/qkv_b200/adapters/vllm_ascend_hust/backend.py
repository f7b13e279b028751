"""The ``get_impl_cls`` dispatcher (the reference's
adapters/vllm_ascend_hust/backend.py:127-158).

Patches the host's ``AscendAttentionBackend.get_impl_cls`` once (idempotent,
marker attribute): ``--kv-cache-dtype int8`` / ``kivi_int4`` (and
``fp8_per_token_head``, on hosts that accept that literal) select the B200
mixins composed over the live host implementation, every other dtype goes to
the original factory. Context parallel is refused for all of them.
"""

from __future__ import annotations

from collections.abc import Callable
from functools import cache
from typing import Any

_DISPATCH_MARKER = "_quantized_kv_plugin_dispatch_installed"
_ORIGINAL_IMPL_GETTER = "_quantized_kv_original_get_impl_cls"
_INT8_CACHE_DTYPE = "int8"
_KIVI_CACHE_DTYPE = "kivi_int4"
_FP8_CACHE_DTYPE = "fp8_per_token_head"


def _require_cache_dtype(expected: str) -> None:
    from vllm.config import get_current_vllm_config

    cache_dtype = get_current_vllm_config().cache_config.cache_dtype
    if cache_dtype != expected:
        raise RuntimeError(
            f"the quantized KV plugin backend {expected!r} is selected only by "
            f"--kv-cache-dtype {expected}; got {cache_dtype!r}"
        )


def _host_attention_v1():
    """``vllm_ascend.attention.attention_v1`` after ``vllm_ascend.ops`` (the
    import order that avoids the host's circular import, backend.py:34-48)."""
    import importlib

    import vllm_ascend.ops  # noqa: F401

    return importlib.import_module("vllm_ascend.attention.attention_v1")


def _context_parallel_enabled() -> bool:
    """``enable_cp()`` or, on newer hosts, ``enable_dcp()`` / ``enable_pcp()``."""
    from vllm_ascend.attention import utils as attention_utils

    enable_cp = getattr(attention_utils, "enable_cp", None)
    if enable_cp is not None:
        return bool(enable_cp())
    split = [getattr(attention_utils, n) for n in ("enable_dcp", "enable_pcp") if hasattr(attention_utils, n)]
    if not split:
        raise RuntimeError(
            "Cannot detect Ascend context parallel: vllm_ascend.attention.utils "
            "exposes neither enable_cp() nor enable_dcp()/enable_pcp()."
        )
    return any(bool(fn()) for fn in split)


@cache
def _build_int8_impl_cls() -> type:
    HostImpl = _host_attention_v1().AscendAttentionBackendImpl
    from ...methods.int8_dynamic.attention_backend import AscendInt8AttentionBackendMixin

    class AscendInt8KvAttentionImpl(AscendInt8AttentionBackendMixin, HostImpl):
        """INT8 dynamic KV impl: B200 kernels over the live host surface."""

    return AscendInt8KvAttentionImpl


@cache
def _build_kivi_impl_cls() -> type:
    HostImpl = _host_attention_v1().AscendAttentionBackendImpl
    from ...methods.kivi_int4.attention_backend import AscendKiviInt4AttentionBackendMixin

    class AscendKiviInt4KvAttentionImpl(AscendKiviInt4AttentionBackendMixin, HostImpl):
        """KIVI INT4 KV impl: B200 kernels over the live host surface."""

        def __init__(self, *args: Any, **kwargs: Any) -> None:
            super().__init__(*args, **kwargs)
            self._init_kivi_state(_KIVI_CACHE_DTYPE, getattr(self, "vllm_config", None))

    return AscendKiviInt4KvAttentionImpl


@cache
def _build_fp8_impl_cls() -> type:
    HostImpl = _host_attention_v1().AscendAttentionBackendImpl
    from ...methods.fp8_per_token_head.attention_backend import AscendFp8PerTokenHeadAttentionBackendMixin

    class AscendFp8PerTokenHeadKvAttentionImpl(AscendFp8PerTokenHeadAttentionBackendMixin, HostImpl):
        """FP8 per-token-head KV impl: B200 kernels over the live host surface."""

    return AscendFp8PerTokenHeadKvAttentionImpl


_IMPL_BUILDERS: dict[str, Callable[[], type]] = {
    _INT8_CACHE_DTYPE: _build_int8_impl_cls,
    _KIVI_CACHE_DTYPE: _build_kivi_impl_cls,
    _FP8_CACHE_DTYPE: _build_fp8_impl_cls,
}


def install_kv_impl_dispatch() -> type:
    """Routes the two quantized cache dtypes to the plugin impls; returns the
    patched host backend class."""
    from vllm.config import get_current_vllm_config

    AscendAttentionBackend = _host_attention_v1().AscendAttentionBackend
    if getattr(AscendAttentionBackend, _DISPATCH_MARKER, False):
        return AscendAttentionBackend
    original = AscendAttentionBackend.get_impl_cls

    def get_impl_cls() -> type:
        cache_dtype = get_current_vllm_config().cache_config.cache_dtype
        builder = _IMPL_BUILDERS.get(cache_dtype)
        if builder is None:
            return original()
        if _context_parallel_enabled():
            raise NotImplementedError(f"Ascend KV cache {cache_dtype} does not support context parallel yet.")
        return builder()

    setattr(AscendAttentionBackend, _ORIGINAL_IMPL_GETTER, original)
    AscendAttentionBackend.get_impl_cls = staticmethod(get_impl_cls)
    setattr(AscendAttentionBackend, _DISPATCH_MARKER, True)
    return AscendAttentionBackend


def _build_backend_cls(cache_dtype: str, class_name: str) -> type:
    AscendAttentionBackend = _host_attention_v1().AscendAttentionBackend

    class AscendKvAttentionBackend(AscendAttentionBackend):
        @staticmethod
        def get_impl_cls() -> type:
            _require_cache_dtype(cache_dtype)
            return _IMPL_BUILDERS[cache_dtype]()

    AscendKvAttentionBackend.__name__ = class_name
    AscendKvAttentionBackend.__qualname__ = class_name
    AscendKvAttentionBackend.__doc__ = f"Backend activated exclusively by ``--kv-cache-dtype {cache_dtype}``."
    return AscendKvAttentionBackend


_BACKENDS_BY_CLASS_NAME = {
    "AscendInt8KvAttentionBackend": _INT8_CACHE_DTYPE,
    "AscendKiviInt4KvAttentionBackend": _KIVI_CACHE_DTYPE,
    "AscendFp8PerTokenHeadKvAttentionBackend": _FP8_CACHE_DTYPE,
}


def __getattr__(name: str) -> Any:
    cache_dtype = _BACKENDS_BY_CLASS_NAME.get(name)
    if cache_dtype is not None:
        return _build_backend_cls(cache_dtype, name)
    raise AttributeError(name)


__all__ = ["install_kv_impl_dispatch"]
