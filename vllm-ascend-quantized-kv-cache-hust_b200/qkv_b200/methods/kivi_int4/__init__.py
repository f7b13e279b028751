"""KIVI INT4 KV cache (``--kv-cache-dtype kivi_int4``): int4 history pages plus
a per-request bf16 residual window. Geometry rules in ``geometry`` (no torch),
the byte layout in ``byte_cache``, the device path in ``attention_backend``."""
