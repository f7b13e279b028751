"""Dynamic per-channel INT8 KV cache (``--kv-cache-dtype int8``).

Metadata registration only (no torch import); the device path is
``attention_backend.AscendInt8AttentionBackendMixin``.
"""

from __future__ import annotations

from ...core.hosts import VLLM_ASCEND_HUST
from ...dtypes import KVQuantMode
from ..base import MethodConfig, MethodSpec
from ..registry import register_method


def _validate_config(config: MethodConfig) -> None:
    """head_size must be a multiple of 8 (methods/int8_dynamic/__init__.py:21-31)."""
    if config.head_size % 8:
        raise ValueError(
            "int8_dynamic expects head_size divisible by 8 for the fused "
            f"attention path, got {config.head_size}"
        )


def _ascend_adapter(method):
    from ...adapters.vllm_ascend_hust import AscendHustAdapter

    return AscendHustAdapter(method)


METHOD_SPEC = register_method(
    MethodSpec(
        name="int8_dynamic",
        dtype="int8",
        summary=(
            "Dynamic per-channel INT8 KV cache: token-axis amax on the first K/V a "
            "layer sees, symmetric zero offset, per-channel antiquant folded into "
            "the B200 paged decode kernel."
        ),
        quant_mode=KVQuantMode.INT8_PER_TENSOR,
        supports=(VLLM_ASCEND_HUST,),
        config_validator=_validate_config,
        adapter_factories={VLLM_ASCEND_HUST: _ascend_adapter},
    )
)

__all__ = ["METHOD_SPEC"]
