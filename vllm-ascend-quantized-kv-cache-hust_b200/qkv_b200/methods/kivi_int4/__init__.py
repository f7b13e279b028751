"""KIVI INT4 KV cache (``--kv-cache-dtype kivi_int4``): int4 history pages plus
a per-request full-precision residual window.

Metadata registration only; geometry rules live in ``geometry`` (no torch),
the byte layout in ``byte_cache``, the device path in ``attention_backend``.
"""

from __future__ import annotations

from ...core.hosts import VLLM_ASCEND_HUST
from ...dtypes import KVQuantMode
from ..base import MethodConfig, MethodSpec
from ..registry import register_method


def _validate_config(config: MethodConfig) -> None:
    from .geometry import validate_kivi_config

    validate_kivi_config(config)


def _ascend_adapter(method):
    from ...adapters.vllm_ascend_hust import AscendHustAdapter

    return AscendHustAdapter(method)


METHOD_SPEC = register_method(
    MethodSpec(
        name="kivi_int4",
        dtype="kivi_int4",
        summary=(
            "KIVI INT4: the last residual_length tokens of a request stay bf16; "
            "older tokens are packed into paged int4 history (keys per channel over "
            "token groups, values per token over head-dim groups) and read by a "
            "fused B200 decode kernel without a dense copy."
        ),
        quant_mode=KVQuantMode.KIVI_INT4,
        supports=(VLLM_ASCEND_HUST,),
        config_validator=_validate_config,
        adapter_factories={VLLM_ASCEND_HUST: _ascend_adapter},
    )
)

__all__ = ["METHOD_SPEC"]
