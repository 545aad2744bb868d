"""Derives the polynomial the attention kernel uses for part of its exp2 evaluations.

Range reduction by the nearest integer (Cody & Waite): 2^x = 2^j * 2^f with
j = rint(x) and f = x - j in [-1/2, 1/2].  rint comes from adding 1.5 * 2^23 in float32
(the sum's low mantissa bits then hold j), so no conversion instruction is needed.
2^f is approximated by p(f) = 1 + c1 f + ... + cn f^n: c0 is pinned to 1 so integer
arguments are exact, and c1..cn minimise the relative error over Chebyshev nodes of
[-1/2, 1/2] by iteratively reweighted least squares (weights pushed toward the error
peaks, approaching equal ripple).  The kernel scales p by 2^j by adding j << 23 to its
bits.  Run to print float32 coefficients and the max relative error of each degree.
"""
import numpy as np


def fit(deg: int, iters: int = 40):
    n = 4000
    f = 0.5 * np.cos(np.pi * (np.arange(n) + 0.5) / n)
    y = np.exp2(f)
    a = np.stack([f ** k for k in range(1, deg + 1)], 1) / y[:, None]
    b = (y - 1.0) / y
    w = np.ones(n)
    for _ in range(iters):
        c, *_ = np.linalg.lstsq(a * w[:, None], b * w, rcond=None)
        rel = np.abs(a @ c - b)
        w = w * (1.0 + 4.0 * rel / rel.max())
    c32 = np.asarray(c, np.float32)
    fine = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
    acc = np.full_like(fine, c32[deg - 1])  # Horner in float32, as the kernel evaluates it
    for k in range(deg - 2, -1, -1):
        acc = acc * fine + c32[k]
    p = acc * fine + np.float32(1.0)
    err = np.max(np.abs(p.astype(np.float64) - np.exp2(fine.astype(np.float64))) / np.exp2(fine))
    return [float(x) for x in c32], float(err)


if __name__ == "__main__":
    for d in (3, 4, 5):
        c, e = fit(d)
        print(d, [f"{x:.9e}" for x in c], f"max rel err {e:.3e}")
