"""Generates the golden fixtures in tests/golden/ by running the REFERENCE.

The reference plugin is pure Python/torch on CPU for everything these fixtures
pin, so this script imports it read-only from the checkout named by its one
argument (or the ``REFERENCE_ROOT`` environment variable) and records what its
own code computes:

* ``int8.npz``      — ``AscendInt8AttentionBackendMixin._prepare_int8_scales``,
  ``_quantize_kv_to_runtime_int8`` and ``_dequant_int8_paged_kv_to_dense``
  (methods/int8_dynamic/attention_backend.py:130-171, :370-404), run on a stub
  layer with the host modules the mixin imports replaced by empty stand-ins.
* ``kivi_pack.npz`` — the six KIVI views written by the reference's
  layout-exact CPU packers (tests/test_kivi_int4.py:703-745, the numerical
  stand-ins of ops/triton/kivi_pack.py) at the five geometries of
  ``GEOMETRIES`` (tests/test_kivi_int4.py:1658-1664), plus tie and
  near-constant-group edge cases and ``kivi_dequant_gather_cache``
  (ops/kivi_gather.py:36-156) over the packed pages.
* ``fp8.npz`` — ``Fp8PerTokenHeadSemantics`` quantise / dequantise / fake
  quant (methods/fp8_per_token_head/semantics.py:52-76) and a store through the
  reference's byte-buffer views (byte_cache.py), with a zero (token, head) and
  E4M3 ties.
* ``kivi_pipeline.npz`` — a multi-request write -> flush -> sync -> gather ->
  attention sequence through ``AscendKiviInt4AttentionBackendMixin.forward``
  (generic branch, methods/kivi_int4/attention_backend.py:1157-1191): bulk
  prefill writes, then decode steps that cross key-window flushes and value
  evictions, one finished request and one roll-back.

Run it where a checkout of the reference exists:
``python tests/golden/make_golden.py <reference checkout> [--only fp8]``. The tests only
read the .npz files it wrote.
"""

from __future__ import annotations

import importlib
import os
import sys
import types
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REFERENCE_ROOT: Path | None = None


def _reference_root() -> Path:
    """The reference checkout: the first argument, else $REFERENCE_ROOT."""
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: make_golden.py <reference checkout> (or set REFERENCE_ROOT)")
    path = Path(root)
    if not (path / "src").is_dir():
        raise SystemExit(f"{path} does not look like a checkout of the reference (no src/)")
    return path


def _import_reference():
    sys.path.insert(0, str(REFERENCE_ROOT / "src"))
    sys.path.insert(0, str(REFERENCE_ROOT / "tests"))
    # stand-ins for the host modules the INT8 mixin imports at module level
    for name in (
        "torch_npu",
        "vllm",
        "vllm.v1",
        "vllm.v1.attention",
        "vllm.v1.attention.backend",
        "vllm_ascend",
        "vllm_ascend.ascend_forward_context",
        "vllm_ascend.attention",
        "vllm_ascend.attention.attention_v1",
    ):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["vllm.v1.attention.backend"].AttentionType = SimpleNamespace(
        ENCODER_DECODER="encoder_decoder"
    )
    sys.modules["vllm_ascend.ascend_forward_context"]._EXTRA_CTX = SimpleNamespace(
        capturing=False
    )
    sys.modules["vllm_ascend.attention.attention_v1"].AscendAttentionState = SimpleNamespace(
        DecodeOnly="DecodeOnly", ChunkedPrefill="ChunkedPrefill", PrefillNoCache="PrefillNoCache"
    )
    int8_ab = importlib.import_module(
        "vllm_ascend_quantized_kv_cache.methods.int8_dynamic.attention_backend"
    )
    kivi_tests = importlib.import_module("test_kivi_int4")
    gather = importlib.import_module("vllm_ascend_quantized_kv_cache.ops.kivi_gather")
    return int8_ab, kivi_tests, gather


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def _kv(gen, tokens, heads, head, outlier_channels, factor, dtype=torch.bfloat16):
    x = torch.randn(tokens, heads, head, generator=gen)
    for h in range(heads):
        for c in outlier_channels[h]:
            x[:, h, c] *= factor
    return x.to(dtype)


# ---------------------------------------------------------------------------
# INT8
# ---------------------------------------------------------------------------


def make_int8(int8_ab) -> dict:
    gen = torch.Generator().manual_seed(1000)
    T, H, D, blk, nb = 64, 8, 128, 16, 4
    outl = [torch.randperm(D, generator=gen)[:4].tolist() for _ in range(H)]
    key = _kv(gen, T, H, D, outl, 20.0)
    value = _kv(gen, T, H, D, outl, 20.0)
    key[:, 3, 7] = 0.0  # an all-zero channel exercises the 1e-12 floor
    value[:, 5, 100] = 0.0

    class Impl(int8_ab.AscendInt8AttentionBackendMixin):
        num_kv_heads = H
        head_size = D

    impl = Impl()
    layer = SimpleNamespace()
    impl._prepare_int8_scales(layer, key, value)
    n_actual = 48
    k8, v8 = impl._quantize_kv_to_runtime_int8(key, value, layer, n_actual)

    # page the first n_actual tokens of two requests (48 + 32) through a
    # shuffled block table, then run the reference dense gather-dequant
    perm = torch.randperm(nb, generator=gen)
    block_table = torch.stack([perm[:2], perm[2:4]]).to(torch.int64)
    seq_lens = [32, 16]
    slots = []
    for b, L in enumerate(seq_lens):
        for p in range(L):
            slots.append(int(block_table[b, p // blk]) * blk + p % blk)
    kc = torch.zeros(nb, blk, H, D, dtype=torch.int8)
    vc = torch.zeros_like(kc)
    slot_t = torch.tensor(slots)
    kc.view(nb * blk, H, D)[slot_t] = k8
    vc.view(nb * blk, H, D)[slot_t] = v8
    impl.key_cache = kc
    dk, dv = impl._dequant_int8_paged_kv_to_dense(
        kc.view(nb, blk, -1), vc.view(nb, blk, -1), block_table, seq_lens, torch.bfloat16, layer
    )
    return {
        "key": _bf16_bits(key),
        "value": _bf16_bits(value),
        "k_inv": _bf16_bits(layer._int8_k_inv_scale.reshape(H, D)),
        "v_inv": _bf16_bits(layer._int8_v_inv_scale.reshape(H, D)),
        "k_aq": _bf16_bits(layer._int8_k_aq_scale.reshape(H, D)),
        "v_aq": _bf16_bits(layer._int8_v_aq_scale.reshape(H, D)),
        "n_actual": np.int64(n_actual),
        "k_codes": k8.numpy(),
        "v_codes": v8.numpy(),
        "slots": np.asarray(slots, np.int64),
        "block_table": block_table.numpy(),
        "seq_lens": np.asarray(seq_lens, np.int64),
        "key_cache": kc.numpy(),
        "value_cache": vc.numpy(),
        "dense_k": _bf16_bits(dk),
        "dense_v": _bf16_bits(dv),
    }


# ---------------------------------------------------------------------------
# KIVI pack + gather at the reference geometries
# ---------------------------------------------------------------------------


def make_kivi_pack(kt, gather) -> dict:
    out = {}
    for gi, (head, kvh, group, block, residual) in enumerate(kt.GEOMETRIES):
        gen = torch.Generator().manual_seed(2000 + gi)
        nb = 3
        tokens = group * (1 if head * kvh >= 1024 else 2)
        outl = [torch.randperm(head, generator=gen)[: max(1, head // 50)].tolist() for _ in range(kvh)]
        key = _kv(gen, tokens, kvh, head, outl, 10.0).to(torch.float32)
        value = _kv(gen, tokens, kvh, head, outl, 1.0).to(torch.float32)
        # edge cases: a constant key group (scale floor) and exact ties
        key[:group, 0, 0] = 0.75
        value[1, 0, :group] = torch.arange(group, dtype=torch.float32) * 0.5
        impl = kt._make_impl(
            residual_length=residual,
            head_size=head,
            num_kv_heads=kvh,
            group_size=group,
            block_size=block,
            num_blocks=nb,
        )
        kt._install_cpu_packers(impl)
        bt = torch.randperm(nb, generator=gen)[:2].view(1, 2).long()
        pos = torch.arange(tokens)
        slots = (bt[0, pos // block] * block + pos % block).long()
        impl._launch_kivi_key_pack(key, slots)
        impl._launch_kivi_value_pack(value, slots)
        small = head * kvh <= 256
        if small:
            gk, gv = gather.kivi_dequant_gather_cache(
                impl.k_quant_cache, impl.k_scale_cache, impl.k_mn_cache,
                impl.v_quant_cache, impl.v_scale_cache, impl.v_mn_cache,
                bt, torch.tensor([tokens - 3]), torch.float32, group,
            )
            gk16, gv16 = gather.kivi_dequant_gather_cache(
                impl.k_quant_cache, impl.k_scale_cache, impl.k_mn_cache,
                impl.v_quant_cache, impl.v_scale_cache, impl.v_mn_cache,
                bt, torch.tensor([tokens - 3]), torch.bfloat16, group,
            )
        p = f"g{gi}_"
        out[p + "geometry"] = np.asarray([head, kvh, group, block, residual, nb], np.int64)
        out[p + "key"] = _bf16_bits(key)
        out[p + "value"] = _bf16_bits(value)
        out[p + "slots"] = slots.numpy()
        out[p + "block_table"] = bt.numpy()
        for name in ("k_quant", "k_scale", "k_mn", "v_quant", "v_scale", "v_mn"):
            out[p + name] = getattr(impl, name + "_cache").numpy()
        if small:
            out[p + "gather_k_f32"] = gk.numpy()
            out[p + "gather_v_f32"] = gv.numpy()
            out[p + "gather_k_bf16"] = _bf16_bits(gk16)
            out[p + "gather_v_bf16"] = _bf16_bits(gv16)
    return out


# ---------------------------------------------------------------------------
# KIVI multi-request pipeline through the mixin's forward()
# ---------------------------------------------------------------------------


def make_kivi_pipeline(kt) -> dict:
    head, kvh, group, block, residual = 64, 2, 16, 32, 32
    num_heads = 4
    nb = 24
    gen = torch.Generator().manual_seed(3000)
    impl = kt._make_impl(
        residual_length=residual,
        max_seqs=4,
        head_size=head,
        num_kv_heads=kvh,
        group_size=group,
        block_size=block,
        num_blocks=nb,
    )
    impl.num_heads = num_heads
    impl.num_queries_per_kv = num_heads // kvh
    impl.scale = head ** -0.5
    kt._install_cpu_packers(impl)

    reqs = ["a", "b", "c"]
    prompt = [45, 64, 100]
    perm = torch.randperm(nb, generator=gen)
    tables = [perm[0:6], perm[6:12], perm[12:18]]
    bt = torch.stack(tables).long()

    def slot(b, pos):
        return int(bt[b, pos // block]) * block + pos % block

    def bf(x):
        return x.to(torch.bfloat16).to(torch.float32)

    rec = {"geometry": np.asarray([head, kvh, group, block, residual, nb, num_heads], np.int64),
           "block_table": bt.numpy()}
    # bulk prefill writes (the PrefillNoCache writer)
    pk, pv = [], []
    for b, n in enumerate(prompt):
        k = bf(torch.randn(n, kvh, head, generator=gen) * 2)
        v = bf(torch.randn(n, kvh, head, generator=gen))
        pk.append(k)
        pv.append(v)
        impl._write_kivi_prefill_cache(
            k, v, torch.tensor([slot(b, p) for p in range(n)]), [reqs[b]], [n]
        )
    rec["prefill_k"] = _bf16_bits(torch.cat(pk))
    rec["prefill_v"] = _bf16_bits(torch.cat(pv))
    rec["prompt_lens"] = np.asarray(prompt, np.int64)

    lens = list(prompt)
    live = [0, 1, 2]
    steps = 40
    step_q, step_k, step_v, step_out, step_meta = [], [], [], [], []
    for s in range(steps):
        finished = None
        if s == 25:  # request c finishes
            finished = {"c"}
            live = [0, 1]
        if s == 30:  # request b is rolled back by 3 tokens before this step
            lens[1] -= 3
        B = len(live)
        for i in live:
            lens[i] += 1
        q = bf(torch.randn(B, num_heads, head, generator=gen))
        k = bf(torch.randn(B, kvh, head, generator=gen) * 2)
        v = bf(torch.randn(B, kvh, head, generator=gen))

        class _State:
            name = "PrefillCacheHit"

        md = SimpleNamespace(
            attn_state=_State(),
            actual_seq_lengths_q=list(range(1, B + 1)),
            seq_lens_list=[lens[i] for i in live],
            slot_mapping=torch.tensor([slot(i, lens[i] - 1) for i in live]),
            block_tables=bt[live],
            req_ids=[reqs[i] for i in live],
            num_actual_tokens=B,
            causal=True,
            finished_req_ids=finished,
        )
        out = torch.zeros(B, num_heads, head)
        impl.forward(None, q, k, v, kt._six_tuple(impl), md, out)
        step_q.append(q.numpy())
        step_k.append(k.numpy())
        step_v.append(v.numpy())
        step_out.append(out.numpy())
        step_meta.append(
            np.asarray(
                [[i, lens[i], slot(i, lens[i] - 1), int(s == 25), int(s == 30)] for i in live], np.int64
            )
        )
    # ragged per-step arrays, padded to 3 rows
    def pad(a, shape):
        o = np.zeros((3,) + shape, np.float32)
        o[: a.shape[0]] = a
        return o

    def bits(a):
        return _bf16_bits(torch.from_numpy(a))

    rec["step_q"] = bits(np.stack([pad(a, (num_heads, head)) for a in step_q]))
    rec["step_k"] = bits(np.stack([pad(a, (kvh, head)) for a in step_k]))
    rec["step_v"] = bits(np.stack([pad(a, (kvh, head)) for a in step_v]))
    rec["step_out"] = np.stack([pad(a, (num_heads, head)) for a in step_out])
    meta = np.full((steps, 3, 5), -1, np.int64)
    for s, m in enumerate(step_meta):
        meta[s, : m.shape[0]] = m
    rec["step_meta"] = meta
    for name in ("k_quant", "k_scale", "k_mn", "v_quant", "v_scale", "v_mn"):
        rec["final_" + name] = getattr(impl, name + "_cache").numpy()
    for b, r in enumerate(reqs):
        for is_key, tag in ((True, "k"), (False, "v")):
            slots, tensors = impl._collect_kivi_residual_window(r, is_key=is_key)
            rec[f"final_win_{tag}_slots_{r}"] = np.asarray(slots, np.int64)
            rec[f"final_win_{tag}_{r}"] = (
                tensors.numpy() if tensors is not None else np.zeros((0, kvh, head), np.float32)
            )
    return rec


def make_fp8() -> dict:
    """``Fp8PerTokenHeadSemantics`` (methods/fp8_per_token_head/semantics.py)
    on bf16 K/V with per-(token, head) magnitudes spanning 1e-3..50, an
    all-zero (token, head) (the 1e-6 scale floor) and exact E4M3 ties, stored
    through the reference's byte-buffer views (byte_cache.py)."""
    from vllm_ascend_quantized_kv_cache.methods.fp8_per_token_head.byte_cache import (
        Fp8PerTokenHeadLayout,
        fp8_caches_from_byte_tensors,
    )
    from vllm_ascend_quantized_kv_cache.methods.fp8_per_token_head.semantics import Fp8PerTokenHeadSemantics

    gen = torch.Generator().manual_seed(1006)
    T, H, D, blk, nb = 40, 4, 64, 16, 4
    mag = torch.exp(torch.empty(T, H, 1).uniform_(-7.0, 4.0, generator=gen))
    key = (torch.randn(T, H, D, generator=gen) * mag).to(torch.bfloat16)
    value = (torch.randn(T, H, D, generator=gen) * mag).to(torch.bfloat16)
    key[5, 1] = 0.0
    # a row whose max is 448 * 2^-k scaled so x / scale lands on E4M3 midpoints
    key[7, 2, :8] = torch.tensor([448.0, 1.0625, 3.0625, 13.0, 0.0029296875, -5.25, 0.5, 2.0 ** -10])
    sem = Fp8PerTokenHeadSemantics(SimpleNamespace(head_size=D))
    kq, ks = sem.quantize(key)
    vq, vs = sem.quantize(value)
    lay = Fp8PerTokenHeadLayout(num_blocks=nb, block_size=blk, num_kv_heads=H, head_size=D)
    kbuf = torch.zeros(nb, blk, H, lay.bytes_per_token_head, dtype=torch.uint8)
    vbuf = torch.zeros_like(kbuf)
    kd, ksc, vd, vsc = fp8_caches_from_byte_tensors(kbuf, vbuf, lay)
    slots = torch.randperm(nb * blk, generator=gen)[:T]
    kd.view(nb * blk, H, D)[slots] = kq.view(torch.uint8)
    ksc.view(nb * blk, H, 1)[slots] = ks
    vd.view(nb * blk, H, D)[slots] = vq.view(torch.uint8)
    vsc.view(nb * blk, H, 1)[slots] = vs
    return {
        "key": _bf16_bits(key),
        "value": _bf16_bits(value),
        "k_codes": kq.view(torch.uint8).numpy(),
        "k_scale": ks.numpy(),
        "v_codes": vq.view(torch.uint8).numpy(),
        "v_scale": vs.numpy(),
        "k_dequant": sem.dequantize(kq, ks).numpy(),
        "v_fake": sem.fake_quant(value).float().numpy(),
        "slots": slots.numpy(),
        "k_buffer": kbuf.numpy(),
        "v_buffer": vbuf.numpy(),
        "geometry": np.array([T, H, D, blk, nb]),
    }


def main() -> None:
    global REFERENCE_ROOT
    args = [a for a in sys.argv[1:]]
    only = None
    if "--only" in args:
        i = args.index("--only")
        only = args[i + 1:i + 2]
        del args[i:i + 2]
    sys.argv[1:] = args
    REFERENCE_ROOT = _reference_root()
    if only and only[0] == "fp8":
        _import_reference()
        np.savez_compressed(HERE / "fp8.npz", **make_fp8())
        print("fp8.npz", (HERE / "fp8.npz").stat().st_size)
        return
    int8_ab, kt, gather = _import_reference()
    torch.manual_seed(0)
    np.savez_compressed(HERE / "int8.npz", **make_int8(int8_ab))
    np.savez_compressed(HERE / "kivi_pack.npz", **make_kivi_pack(kt, gather))
    np.savez_compressed(HERE / "kivi_pipeline.npz", **make_kivi_pipeline(kt))
    np.savez_compressed(HERE / "fp8.npz", **make_fp8())
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
