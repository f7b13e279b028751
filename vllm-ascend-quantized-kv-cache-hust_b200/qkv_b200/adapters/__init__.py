"""Host integration (vllm-ascend-hust): the ``get_impl_cls`` dispatcher."""
