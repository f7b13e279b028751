"""Quantisation methods; importing this package registers their metadata only."""

from . import fp8_per_token_head, int8_dynamic, kivi_int4  # noqa: F401  (registration side effect)

__all__ = ["fp8_per_token_head", "int8_dynamic", "kivi_int4"]
