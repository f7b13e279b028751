"""qkv_b200 — B200 (sm_100a) implementation of the quantized-KV attention path
of the vllm-ascend-quantized-kv-cache plugin (``--kv-cache-dtype int8`` and
``kivi_int4``).

Importing the package is lazy: no torch, vllm or device module is loaded until
a method's device path or a host adapter is used. The kernels live in
``libqkv_sm100.so`` (C ABI: include/qkv_sm100.h) and are reached through
``qkv_b200.ops``.

    from qkv_b200 import kv_methods
    kv_methods.list()
    kv_methods.get("kivi_int4", group_size=64).resolve_layout()
    kv_methods.activate("kivi_int4", host="vllm_ascend_hust")
"""

from ._version import __version__
from .core import VLLM_ASCEND_HUST
from .dtypes import KVCacheLayout, KVQuantMode, get_kv_quant_mode, is_quantized_kv_cache, resolve_layout
from .methods.base import KvQuantMethod


def _load_methods() -> None:
    from . import methods  # noqa: F401  (registration side effect)


class _KvMethodsFacade:
    """Discovery / configuration / activation API (the reference's facade,
    __init__.py:54-108)."""

    @staticmethod
    def get(name: str, **config) -> KvQuantMethod:
        _load_methods()
        from .methods.registry import get_method

        return get_method(name, **config)

    @staticmethod
    def list(host: str | None = None) -> list[str]:
        _load_methods()
        from .methods.registry import list_methods

        return list(list_methods(host))

    @staticmethod
    def describe(name: str) -> dict:
        _load_methods()
        from .methods.registry import get_spec

        return get_spec(name).describe()

    @staticmethod
    def activate(name: str, *, host: str | None = None, **config) -> dict:
        _load_methods()
        from .core.activation import activate as _activate

        return _activate(name, host=host, **config)


kv_methods = _KvMethodsFacade()

__all__ = [
    "KVCacheLayout",
    "KVQuantMode",
    "KvQuantMethod",
    "VLLM_ASCEND_HUST",
    "__version__",
    "get_kv_quant_mode",
    "is_quantized_kv_cache",
    "kv_methods",
    "resolve_layout",
]
