"""``vllm.general_plugins`` entry point (contract of the reference's
bootstrap.py:20-35): called by vLLM at start-up.

With the Ascend host stack importable it installs the ``get_impl_cls``
dispatcher and reports the two selectable methods; anywhere else it changes
nothing and returns ``[]``. Installing the dispatcher selects nothing by
itself: ``--kv-cache-dtype int8`` or ``kivi_int4`` does.
"""

from __future__ import annotations

import importlib.util

REGISTERED_METHODS = ("int8_dynamic", "kivi_int4")
HOST_MODULE = "vllm_ascend"


def host_stack_present() -> bool:
    """Whether the vllm-ascend-hust host can be imported (looked up, not
    imported)."""
    try:
        return importlib.util.find_spec(HOST_MODULE) is not None
    except (ImportError, ValueError):
        return False


def register_plugins() -> list[str]:
    if not host_stack_present():
        return []
    from .adapters.vllm_ascend_hust.backend import install_kv_impl_dispatch

    install_kv_impl_dispatch()
    print(
        "[qkv_b200] quantized KV attention installed; select it with --kv-cache-dtype int8 or kivi_int4",
        flush=True,
    )
    return list(REGISTERED_METHODS)


__all__ = ["REGISTERED_METHODS", "host_stack_present", "register_plugins"]
