"""The quantized KV cache methods: ``int8_dynamic`` (``--kv-cache-dtype
int8``), ``kivi_int4`` and ``fp8_per_token_head``; each package holds the
attention mixin and its layout rules. Importing this package imports none of
them (and no torch)."""
