"""FP8 per-token-head KV cache (``fp8_per_token_head``): E4M3 codes with one
fp32 scale per (token, head), computed online at write time.

Metadata registration only (no torch import). The reference registers the
method's contract but wires no adapter and keeps it out of its selectable
methods (no read path); here the device path exists
(``attention_backend.AscendFp8PerTokenHeadAttentionBackendMixin``), the
adapter is wired and the ``get_impl_cls`` dispatcher routes the literal when a
host's config carries it. ``bootstrap.REGISTERED_METHODS`` keeps the
reference's two methods.
"""

from __future__ import annotations

from ...core.hosts import VLLM_ASCEND_HUST
from ...dtypes import KVQuantMode
from ..base import MethodConfig, MethodSpec
from ..registry import register_method


def _validate_config(config: MethodConfig) -> None:
    """head_size a positive multiple of 4 (fp32 scale alignment)."""
    if config.head_size <= 0 or config.head_size % 4:
        raise ValueError(
            "fp8_per_token_head requires head_size positive and divisible "
            f"by 4 (fp32 scale alignment), got {config.head_size}"
        )


def _ascend_adapter(method):
    from ...adapters.vllm_ascend_hust import AscendHustAdapter

    return AscendHustAdapter(method)


METHOD_SPEC = register_method(
    MethodSpec(
        name="fp8_per_token_head",
        dtype="fp8_per_token_head",
        summary=(
            "Per-token-head dynamic-scale E4M3 storage: each (token, head) keeps head_size E4M3 bytes plus one "
            "fp32 scale computed at write time; B200 store, paged decode and dense-gather kernels."
        ),
        quant_mode=KVQuantMode.FP8_PER_TOKEN_HEAD,
        supports=(VLLM_ASCEND_HUST,),
        config_validator=_validate_config,
        adapter_factories={VLLM_ASCEND_HUST: _ascend_adapter},
    )
)

__all__ = ["METHOD_SPEC"]
