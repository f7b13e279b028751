"""Device ops of qkv_b200: thin torch wrappers over libqkv_sm100.so.

Every op validates on the host (the reference's validators and messages) and
launches one of the sm_100a kernels on the current CUDA stream; none has a CPU
fallback.
"""

from .fp8 import fp8_dequant_gather, fp8_paged_decode, fp8_store
from .int8 import int8_calc_scales, int8_dequant_gather, int8_paged_decode, int8_quant_store
from .kivi_decode import kivi_paged_decode
from .kivi_gather import kivi_dequant_gather
from .kivi_pack import kivi_pack_key_cache, kivi_pack_kv_cache, kivi_pack_value_cache
from .prefill import dense_prefill

__all__ = [
    "dense_prefill",
    "fp8_dequant_gather",
    "fp8_paged_decode",
    "fp8_store",
    "int8_calc_scales",
    "int8_dequant_gather",
    "int8_paged_decode",
    "int8_quant_store",
    "kivi_dequant_gather",
    "kivi_pack_key_cache",
    "kivi_pack_kv_cache",
    "kivi_pack_value_cache",
    "kivi_paged_decode",
]
