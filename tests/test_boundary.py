"""The reference-facing surface: dtype contract, KIVI geometry rules,
bootstrap, the get_impl_cls dispatcher and the KIVI byte budget / six-view
split — the behaviour the reference's tests/test_plugin.py and
tests/test_kivi_int4.py:1205-1400 pin."""

from __future__ import annotations

import subprocess
import sys
from types import SimpleNamespace

import pytest
import torch

from qkv_b200 import KVQuantMode, bootstrap, resolve_layout
from qkv_b200.methods.kivi_int4.byte_cache import (
    KiviByteCacheLayout,
    kivi_byte_cache_layout,
    kivi_caches_from_byte_tensors,
)
from qkv_b200.methods.kivi_int4.geometry import validate_kivi_config, validate_kivi_geometry


def test_layout_contract():
    assert resolve_layout("int8", 128).storage_dtype == "int8"
    lay = resolve_layout("kivi_int4", 128)
    assert lay.storage_dtype == "uint8" and lay.packed_last_dim == 64
    assert lay.quant_mode is KVQuantMode.KIVI_INT4
    assert resolve_layout("fp8_per_token_head", 128).storage_dtype == "uint8"
    with pytest.raises(ValueError, match="positive even"):
        resolve_layout("kivi_int4", 127)
    with pytest.raises(ValueError, match="not a registered"):
        resolve_layout("int4", 128)


@pytest.mark.parametrize(
    "overrides, match",
    [
        ({"group_size": 7}, "divisible by 8"),
        ({"residual_length": 4, "group_size": 8}, "residual_length"),
        ({"head_size": 12}, "head_size"),
        ({"head_size": 8, "group_size": 16}, "head_size"),
        ({"block_size": 8, "group_size": 16}, "block_size"),
    ],
)
def test_geometry_rejects(overrides, match):
    kw = dict(head_size=32, group_size=8, residual_length=16, block_size=16)
    kw.update(overrides)
    with pytest.raises(ValueError, match=match):
        validate_kivi_geometry(**kw)
    with pytest.raises(ValueError, match=match):
        validate_kivi_config(SimpleNamespace(**kw))
    # a live impl carries the kivi_* names
    impl = SimpleNamespace(head_size=kw["head_size"], kivi_group_size=kw["group_size"],
                           kivi_residual_length=kw["residual_length"], block_size=kw["block_size"])
    with pytest.raises(ValueError, match=match):
        validate_kivi_config(impl)


def test_import_needs_no_torch():
    code = "import sys; import qkv_b200, qkv_b200.bootstrap, qkv_b200.methods; print('torch' in sys.modules)"
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         env={"PYTHONPATH": ":".join(sys.path)})
    assert out.stdout.strip() == "False", out.stderr


def test_bootstrap_noop_without_host(monkeypatch):
    monkeypatch.setattr(bootstrap, "host_stack_present", lambda: False)
    assert bootstrap.register_plugins() == []


def test_bootstrap_installs_the_dispatcher(monkeypatch):
    calls = []
    monkeypatch.setattr(bootstrap, "host_stack_present", lambda: True)
    import qkv_b200.adapters.vllm_ascend_hust.backend as backend

    monkeypatch.setattr(backend, "install_kv_impl_dispatch", lambda: calls.append("install"))
    assert bootstrap.register_plugins() == ["int8_dynamic", "kivi_int4"]
    assert calls == ["install"]


@pytest.fixture
def host_stack(monkeypatch):
    import importlib.machinery
    import types

    def stub(name):
        m = types.ModuleType(name)
        m.__spec__ = importlib.machinery.ModuleSpec(name, None)
        monkeypatch.setitem(sys.modules, name, m)
        return m

    for n in ("vllm", "vllm_ascend", "vllm_ascend.attention", "vllm_ascend.ops"):
        stub(n)
    vcfg = stub("vllm.config")
    av1 = stub("vllm_ascend.attention.attention_v1")
    utils = stub("vllm_ascend.attention.utils")

    class HostImpl:
        def __init__(self, *a, **k):
            self.num_heads = 4
            self.num_kv_heads = 2
            self.head_size = 32
            self.num_queries_per_kv = 2
            self.scale = 0.125
            self.vllm_config = SimpleNamespace(
                cache_config=SimpleNamespace(kivi_group_size=8, kivi_residual_length=16),
                scheduler_config=SimpleNamespace(max_num_seqs=3),
            )

    class HostBackend:
        @staticmethod
        def get_impl_cls():
            return HostImpl

    av1.AscendAttentionBackend = HostBackend
    av1.AscendAttentionBackendImpl = HostImpl
    cc = SimpleNamespace(cache_dtype="auto")
    vcfg.get_current_vllm_config = lambda: SimpleNamespace(cache_config=cc)
    utils.enable_cp = lambda: False
    from qkv_b200.adapters.vllm_ascend_hust import backend

    backend.impl_class.cache_clear()
    yield SimpleNamespace(backend=HostBackend, impl=HostImpl, cc=cc, utils=utils, install=backend.install_kv_impl_dispatch)
    backend.impl_class.cache_clear()


def test_dispatch_selects_plugin_only_for_quantized_dtypes(host_stack):
    be = host_stack.backend
    assert host_stack.install() is be
    assert be._quantized_kv_plugin_dispatch_installed
    assert be._quantized_kv_original_get_impl_cls() is host_stack.impl
    assert be.get_impl_cls() is host_stack.impl
    host_stack.cc.cache_dtype = "kivi_int4"
    cls = be.get_impl_cls()
    from qkv_b200.methods.kivi_int4.attention_backend import AscendKiviInt4AttentionBackendMixin

    assert issubclass(cls, AscendKiviInt4AttentionBackendMixin) and issubclass(cls, host_stack.impl)
    impl = cls()
    assert impl.enable_kivi and impl.kivi_group_size == 8 and impl.kivi_residual_length == 16
    assert impl.kivi_max_num_seqs == 3
    host_stack.cc.cache_dtype = "int8"
    from qkv_b200.methods.int8_dynamic.attention_backend import AscendInt8AttentionBackendMixin

    assert issubclass(be.get_impl_cls(), AscendInt8AttentionBackendMixin)
    host_stack.cc.cache_dtype = "fp8_per_token_head"
    from qkv_b200.methods.fp8_per_token_head.attention_backend import AscendFp8PerTokenHeadAttentionBackendMixin

    assert issubclass(be.get_impl_cls(), AscendFp8PerTokenHeadAttentionBackendMixin)
    # idempotent install
    wrapped = be.get_impl_cls
    assert host_stack.install() is be and be.get_impl_cls is wrapped
    host_stack.cc.cache_dtype = "auto"
    assert be.get_impl_cls() is host_stack.impl


def test_dispatch_refuses_context_parallel(host_stack):
    host_stack.install()
    host_stack.utils.enable_cp = lambda: True
    host_stack.cc.cache_dtype = "kivi_int4"
    with pytest.raises(NotImplementedError, match="does not support context parallel"):
        host_stack.backend.get_impl_cls()
    host_stack.cc.cache_dtype = "auto"
    assert host_stack.backend.get_impl_cls() is host_stack.impl


# ---------------------------------------------------------------- byte cache


def test_byte_budget_and_compression():
    lay = KiviByteCacheLayout(num_blocks=1, block_size=128, num_kv_heads=8, head_size=128, group_size=128)
    assert lay.bytes_per_token_head == 72
    assert lay.compression_vs_fp16() == pytest.approx(256 / 72)
    assert lay.page_size_bytes() == 2 * 128 * 8 * 72
    assert KiviByteCacheLayout(num_blocks=1, block_size=128, num_kv_heads=8, head_size=128,
                               group_size=64).bytes_per_token_head == 80


@pytest.mark.parametrize("head,group,block,kvh,nb", [(128, 128, 128, 8, 7), (32, 8, 16, 2, 3), (64, 32, 256, 4, 2)])
def test_host_buffers_rebuild_the_layout_and_alias(head, group, block, kvh, nb):
    lay = KiviByteCacheLayout(num_blocks=nb, block_size=block, num_kv_heads=kvh, head_size=head, group_size=group)
    raw = torch.zeros((2, nb, block, kvh, lay.bytes_per_token_head), dtype=torch.uint8)
    assert lay.page_size_bytes() * nb == 2 * lay.region_bytes
    assert kivi_byte_cache_layout(raw[0], raw[1], num_kv_heads=kvh, head_size=head, group_size=group) == lay
    kq, ks, km, vq, vs, vm = kivi_caches_from_byte_tensors(raw[0], raw[1], lay)
    assert kq.shape == (nb, kvh, head, block // 8) and kq.dtype == torch.int32
    assert vq.shape == (nb, block, kvh, head // 8)
    ks[0, 0, 0, 0] = 3.5
    assert float(raw[0].reshape(-1).view(torch.float32)[kq.numel()]) == 3.5
    kq[0, 0, 0, 0] = 0x04030201
    assert raw[0].reshape(-1)[:4].tolist() == [1, 2, 3, 4]


def test_byte_cache_rejects_bad_buffers():
    lay = KiviByteCacheLayout(num_blocks=4, block_size=16, num_kv_heads=2, head_size=32, group_size=8)
    k = torch.zeros(4, 16, 2, lay.bytes_per_token_head, dtype=torch.uint8)
    v = torch.zeros_like(k)
    with pytest.raises(RuntimeError, match="equal regions"):
        kivi_byte_cache_layout(k, v[:1], num_kv_heads=2, head_size=32, group_size=8)
    with pytest.raises(RuntimeError, match="must be contiguous"):
        kivi_byte_cache_layout(k.transpose(0, 1), v, num_kv_heads=2, head_size=32, group_size=8)
    with pytest.raises(RuntimeError, match="value cache must hold"):
        kivi_caches_from_byte_tensors(k, v[:-1], lay)
    dense = torch.zeros(4, 16, 2, 32, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="must hold|whole number of pages"):
        kivi_byte_cache_layout(dense, dense.clone(), num_kv_heads=2, head_size=32, group_size=8)


def test_mixin_binds_one_host_allocation_of_both_sides():
    """The host allocator's single (2, NB, block, KVH, S) uint8 tensor binds
    like the 2-tuple of its halves: the six views alias it."""
    from types import SimpleNamespace

    from qkv_b200.methods.kivi_int4.attention_backend import AscendKiviInt4AttentionBackendMixin

    class Impl(AscendKiviInt4AttentionBackendMixin):
        num_heads, num_kv_heads, head_size, num_queries_per_kv, scale = 4, 2, 32, 2, 0.125

    impl = Impl()
    impl._init_kivi_state("kivi_int4", SimpleNamespace(
        cache_config=SimpleNamespace(kivi_group_size=8, kivi_residual_length=16),
        scheduler_config=SimpleNamespace(max_num_seqs=2)))
    lay = KiviByteCacheLayout(num_blocks=3, block_size=16, num_kv_heads=2, head_size=32, group_size=8)
    raw = torch.zeros((2, 3, 16, 2, lay.bytes_per_token_head), dtype=torch.uint8)
    impl._bind_kivi_cache(raw)
    assert impl.k_quant_cache.shape == (3, 2, 32, 2) and impl.v_quant_cache.shape == (3, 16, 2, 4)
    impl.v_quant_cache[0, 0, 0, 0] = 0x01020304
    assert raw[1].reshape(-1)[:4].tolist() == [4, 3, 2, 1]
    assert lay.page_size_bytes() * 3 == raw.numel()
