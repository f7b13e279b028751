"""The ``get_impl_cls`` dispatcher (contract of the reference's
adapters/vllm_ascend_hust/backend.py:127-158).

``install_kv_impl_dispatch()`` wraps the host's
``AscendAttentionBackend.get_impl_cls`` once: the wrapped factory reads the
running config's ``cache_config.cache_dtype`` and, for a quantized literal,
returns this package's attention mixin composed over the live host impl
class (built once per literal); every other literal goes to the host's own
factory. Context parallel is refused for the quantized literals. The marker
and original-getter attribute names, the refusal message and the idempotence
are the host contract.
"""

from __future__ import annotations

import functools
import importlib

_DISPATCH_MARKER = "_quantized_kv_plugin_dispatch_installed"
_ORIGINAL_IMPL_GETTER = "_quantized_kv_original_get_impl_cls"

# cache dtype literal -> (module of the mixin, mixin class, composed class name)
_METHODS = {
    "int8": ("int8_dynamic", "AscendInt8AttentionBackendMixin", "AscendInt8KvAttentionImpl"),
    "kivi_int4": ("kivi_int4", "AscendKiviInt4AttentionBackendMixin", "AscendKiviInt4KvAttentionImpl"),
    "fp8_per_token_head": (
        "fp8_per_token_head", "AscendFp8PerTokenHeadAttentionBackendMixin", "AscendFp8PerTokenHeadKvAttentionImpl"
    ),
}


def _attention_v1():
    # vllm_ascend.ops first: importing attention_v1 on its own runs into the
    # host's circular import
    importlib.import_module("vllm_ascend.ops")
    return importlib.import_module("vllm_ascend.attention.attention_v1")


def _cache_dtype() -> str:
    from vllm.config import get_current_vllm_config

    return get_current_vllm_config().cache_config.cache_dtype


def _context_parallel() -> bool:
    """The host's context-parallel switch: ``enable_cp()``, or on hosts that
    split it, ``enable_dcp()`` / ``enable_pcp()``; a host with none of them
    cannot be checked and is refused."""
    utils = importlib.import_module("vllm_ascend.attention.utils")
    probes = [getattr(utils, n) for n in ("enable_cp",) if hasattr(utils, n)]
    probes = probes or [getattr(utils, n) for n in ("enable_dcp", "enable_pcp") if hasattr(utils, n)]
    if not probes:
        raise RuntimeError(
            "Cannot detect Ascend context parallel: vllm_ascend.attention.utils "
            "exposes neither enable_cp() nor enable_dcp()/enable_pcp()."
        )
    return any(bool(p()) for p in probes)


@functools.cache
def impl_class(cache_dtype: str) -> type:
    """The mixin of ``cache_dtype`` composed over the host's
    ``AscendAttentionBackendImpl`` (one class per literal and process)."""
    package, mixin_name, class_name = _METHODS[cache_dtype]
    mixin = getattr(importlib.import_module(f"qkv_b200.methods.{package}.attention_backend"), mixin_name)
    host_impl = _attention_v1().AscendAttentionBackendImpl
    cls = type(class_name, (mixin, host_impl),
               {"__doc__": f"--kv-cache-dtype {cache_dtype}: B200 kernels over the live host impl."})
    if cache_dtype == "kivi_int4":
        def __init__(self, *args, **kwargs):  # the KIVI state reads the host ctor's vllm_config
            super(cls, self).__init__(*args, **kwargs)
            self._init_kivi_state(cache_dtype, getattr(self, "vllm_config", None))

        cls.__init__ = __init__
    return cls


def install_kv_impl_dispatch() -> type:
    """Installs the dispatcher (once; later calls change nothing) and returns
    the host backend class."""
    backend = _attention_v1().AscendAttentionBackend
    if getattr(backend, _DISPATCH_MARKER, False):
        return backend
    host_factory = backend.get_impl_cls

    def get_impl_cls() -> type:
        cache_dtype = _cache_dtype()
        if cache_dtype not in _METHODS:
            return host_factory()
        if _context_parallel():
            raise NotImplementedError(f"Ascend KV cache {cache_dtype} does not support context parallel yet.")
        return impl_class(cache_dtype)

    setattr(backend, _ORIGINAL_IMPL_GETTER, host_factory)
    backend.get_impl_cls = staticmethod(get_impl_cls)
    setattr(backend, _DISPATCH_MARKER, True)
    return backend


__all__ = ["impl_class", "install_kv_impl_dispatch"]
