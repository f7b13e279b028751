"""qkv_b200 — B200 (sm_100a) implementation of the quantized-KV attention path
of the vllm-ascend-quantized-kv-cache plugin (``--kv-cache-dtype int8`` and
``kivi_int4``).

The host entry is ``qkv_b200.bootstrap.register_plugins`` (the
``vllm.general_plugins`` entry point), which installs the ``get_impl_cls``
dispatcher. Importing the package loads no torch, vllm or device module; the
kernels live in ``libqkv_sm100.so`` (C ABI: include/qkv_sm100.h) and are
reached through ``qkv_b200.ops``.
"""

from ._version import __version__
from .dtypes import KVCacheLayout, KVQuantMode, get_kv_quant_mode, is_quantized_kv_cache, resolve_layout

__all__ = [
    "KVCacheLayout",
    "KVQuantMode",
    "__version__",
    "get_kv_quant_mode",
    "is_quantized_kv_cache",
    "resolve_layout",
]
