"""The FMA-pipe exponential of the tcgen05 prompt attention (``exp2_fma2`` in
``csrc/prefill_tc.cu``), checked on the CPU: its coefficients are the ones the
committed fit produces, and a float32 restatement of its steps (the 1.5 * 2^23
rounding shift, the cubic, the exponent-field add, zero below -126) stays
within the fit's relative error over every argument the softmax can give it."""

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
    x = x.astype(np.float32)
    rnd = np.float32(12582912.0)
    t = (x + rnd).astype(np.float32)
    f = (x - (t - rnd).astype(np.float32)).astype(np.float32)
    q = _fma_f32(np.full_like(f, c[3]), f, np.full_like(f, c[2]))
    q = _fma_f32(q, f, np.full_like(f, c[1]))
    q = _fma_f32(q, f, np.full_like(f, c[0]))
    with np.errstate(invalid="ignore"):
        bits = q.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)
        p = (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
        return np.where(x >= np.float32(-126.0), p, np.float32(0.0))


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


def test_fma_pipe_exp2_masked_and_underflowing_scores_give_zero():
    """Below -126 (masked scores are -inf) the result is 0, as the SFU's
    flush-to-zero ex2 gives, so a row that sees no key keeps a zero sum."""
    c = _kernel_coefficients()
    with np.errstate(invalid="ignore", over="ignore"):
        got = _exp2_fma2(np.array([-np.inf, -1e30, -1000.0, -200.0, -126.5, -126.01], dtype=np.float32), c)
    assert np.all(got == 0.0), got
    edge = _exp2_fma2(np.array([-125.5, -125.0], dtype=np.float32), c).astype(np.float64)
    assert np.all(np.abs(edge / np.exp2([-125.5, -125.0]) - 1.0) < 1e-4), edge
    # at -126 itself the result may be subnormal (a cubic value below 1 at
    # exponent -126): still about 2^-126
    last = float(_exp2_fma2(np.array([-126.0], dtype=np.float32), c)[0])
    assert abs(last / 2.0 ** -126 - 1.0) < 1e-3, last
