"""Coefficients of the cubic behind ``exp2_fma2`` in ``prefill_tc.cu``.

A relative-error minimax fit of 2^f on [-1/2, 1/2] by Lawson's algorithm
(iteratively reweighted least squares: each pass reweights the Chebyshev-spaced
sample points by their current relative error, which drives the weighted
least-squares solution toward the equal-ripple minimax one). Prints the four
float32 coefficients (constant term first) and the largest relative error of
the cubic evaluated in float32 Horner form, the way the kernel evaluates it.
"""
import numpy as np

DEG = 3


def fit(deg=DEG, points=4001, passes=200):
    x = np.cos(np.linspace(0.0, np.pi, points)) * 0.5
    y = np.exp2(x)
    v = np.vander(x, deg + 1, increasing=True)
    w = np.ones_like(x)
    c = None
    for _ in range(passes):
        sw = np.sqrt(w) / y
        c, *_ = np.linalg.lstsq(v * sw[:, None], y * sw, rcond=None)
        w = w * np.abs((v @ c - y) / y)
        w /= w.sum()
    return np.asarray(c, dtype=np.float32)


def horner_f32(c, f):
    q = np.float32(c[-1]) * np.ones_like(f, dtype=np.float32)
    for k in range(len(c) - 2, -1, -1):
        q = (q * f + np.float32(c[k])).astype(np.float32)
    return q


def max_rel_error(c):
    f = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
    return float(np.max(np.abs(horner_f32(c, f).astype(np.float64) / np.exp2(f.astype(np.float64)) - 1.0)))


if __name__ == "__main__":
    c = fit()
    print("coefficients", [float(v) for v in c])
    print("max relative error (float32 Horner)", max_rel_error(c))
