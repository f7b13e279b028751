"""``vllm.general_plugins`` entry point (the reference's bootstrap.py:20-35).

Installed as a plugin, vLLM calls ``register_plugins()`` at start-up: on the
Ascend host stack it activates both methods (installs the ``get_impl_cls``
dispatcher); anywhere else it is a no-op. Registration alone changes nothing:
``--kv-cache-dtype int8`` or ``kivi_int4`` selects an implementation.
"""

from __future__ import annotations

from .core.hosts import VLLM_ASCEND_HUST, detect_host

REGISTERED_METHODS = ("int8_dynamic", "kivi_int4")


def register_plugins() -> list[str]:
    if detect_host() != VLLM_ASCEND_HUST:
        return []
    from .core.activation import activate

    for name in REGISTERED_METHODS:
        activate(name, host=VLLM_ASCEND_HUST)
    print(
        "[qkv_b200] registered quantized KV attention backends; enable one with "
        f"--kv-cache-dtype {', '.join(('int8', 'kivi_int4'))}",
        flush=True,
    )
    return list(REGISTERED_METHODS)


__all__ = ["REGISTERED_METHODS", "detect_host", "register_plugins"]
