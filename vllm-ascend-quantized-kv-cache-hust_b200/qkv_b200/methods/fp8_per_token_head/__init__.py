"""FP8 per-token-head KV cache (``fp8_per_token_head``): E4M3 codes with one
fp32 scale per (token, head), computed at write time. The reference registers
this method's contract without a read path; here the device path exists
(``attention_backend.AscendFp8PerTokenHeadAttentionBackendMixin``) and the
``get_impl_cls`` dispatcher routes the literal when a host's config carries
it. ``bootstrap.REGISTERED_METHODS`` keeps the reference's two methods."""
