"""Derives the exp2 polynomial used by the prefill softmax (gqa_prefill.cu).

2^f on f in [-1/2, 1/2] by a degree-3 polynomial with minimal maximum
relative error, found with Lawson's algorithm (iteratively reweighted least
squares on a dense grid), then rounded to float32.  Prints the coefficients
and the relative error of the float32 Horner evaluation.
"""
import numpy as np


def fit(degree=3, n=20001, iters=200):
    f = np.linspace(-0.5, 0.5, n)
    y = np.exp2(f)
    v = np.vander(f, degree + 1, increasing=True) / y[:, None]
    w = np.ones_like(f)
    for _ in range(iters):
        sw = np.sqrt(w)
        c, *_ = np.linalg.lstsq(v * sw[:, None], sw, rcond=None)
        w = w * np.abs(v @ c - 1)
        w /= w.sum()
    return c.astype(np.float32)


def horner_f32(c, f):
    f = np.asarray(f, dtype=np.float32)
    r = np.full_like(f, c[-1])
    for k in range(len(c) - 2, -1, -1):
        r = (r.astype(np.float64) * f + np.float64(c[k])).astype(np.float32)  # one rounding, as fma
    return r


if __name__ == "__main__":
    c = fit()
    xs = np.linspace(-0.5, 0.5, 200001, dtype=np.float32)
    err = np.abs(horner_f32(c, xs).astype(np.float64) / np.exp2(xs.astype(np.float64)) - 1).max()
    for k, v in enumerate(c):
        print(f"kExp2C{k} = {float(v)!r}f")
    print(f"max relative error {err:.3g}")
