"""Dynamic per-channel INT8 KV cache (``--kv-cache-dtype int8``): the device
path is ``attention_backend.AscendInt8AttentionBackendMixin``."""
