"""The FMA-pipe exponential of the tcgen05 prompt attention (``exp2_fma2`` in
``csrc/prefill_tc.cu``), checked on the CPU: its coefficients are the ones the
committed fit produces, and a float32 restatement of its steps (clamp, the
1.5 * 2^23 rounding shift, the cubic, the exponent-field add) stays within the
fit's relative error over every argument the softmax can give it."""

from __future__ import annotations

import importlib.util
import re

import numpy as np

from conftest import PKG

CSRC = PKG / "csrc"


def _fit_module():
    spec = importlib.util.spec_from_file_location("exp2_poly_fit", CSRC / "exp2_poly_fit.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _kernel_coefficients():
    src = (CSRC / "prefill_tc.cu").read_text()
    found = dict(re.findall(r"kExp2C(\d) = ([0-9.eE+-]+)f", src))
    assert sorted(found) == ["0", "1", "2", "3"], found
    return np.array([float(found[str(k)]) for k in range(4)], dtype=np.float32)


def _fma_f32(a, b, c):
    # one rounding, as fma.rn.f32 (the float64 product of two float32 is exact)
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def _exp2_fma2(x, c):
    """float32 restatement of exp2_fma2, one lane."""
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    rnd = np.float32(12582912.0)
    t = (x + rnd).astype(np.float32)
    f = (x - (t - rnd).astype(np.float32)).astype(np.float32)
    q = _fma_f32(np.full_like(f, c[3]), f, np.full_like(f, c[2]))
    q = _fma_f32(q, f, np.full_like(f, c[1]))
    q = _fma_f32(q, f, np.full_like(f, c[0]))
    bits = q.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def test_kernel_coefficients_are_the_committed_fit():
    fit = _fit_module()
    c = fit.fit()
    np.testing.assert_array_equal(_kernel_coefficients(), c)
    assert fit.max_rel_error(c) < 1e-4


def test_fma_pipe_exp2_relative_error_over_softmax_arguments():
    c = _kernel_coefficients()
    # the softmax's arguments: scores minus a lazy running max, so at most
    # a few log2 units above 0 and as low as the exponent range allows
    x = np.concatenate([np.linspace(-125.0, 9.0, 400001), np.arange(-125, 10) + 0.5,
                        np.arange(-125, 10).astype(np.float64)]).astype(np.float32)
    got = _exp2_fma2(x, c).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert rel.max() < 1e-4, (float(rel.max()), float(x[np.argmax(rel)]))


def test_fma_pipe_exp2_masked_and_underflowing_scores_stay_negligible():
    c = _kernel_coefficients()
    x = np.array([-np.inf, -1e30, -1000.0, -200.0, -126.0, -125.9], dtype=np.float32)
    got = _exp2_fma2(x, c).astype(np.float64)
    assert np.all(np.isfinite(got)) and np.all(got >= 0.0)
    assert np.all(got <= 2.0 ** -125), got
