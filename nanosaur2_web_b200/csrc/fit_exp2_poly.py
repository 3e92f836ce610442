"""Fit the polynomial behind the FMA-pipe exp2 of attention.cu (run offline, prints coefficients).

2^x is split as 2^n * 2^f with n = round(x) and f = x - n in [-0.5, 0.5]; 2^f is approximated by a
degree-3 polynomial whose maximum relative error on [-0.5, 0.5] is minimised by Lawson's iteratively
reweighted least squares (a standard route to the minimax / Chebyshev-equioscillation fit).
The fit gives a maximum relative error of 8.4e-5, far below the 2^-9 relative rounding of the bf16
probabilities it feeds.
"""

import numpy as np


def fit(deg=3, iters=200):
    f = np.linspace(-0.5, 0.5, 200001)
    y = np.exp2(f)
    A = np.vander(f, deg + 1, increasing=True)
    w = np.ones_like(f)
    for _ in range(iters):
        W = w / y
        c, *_ = np.linalg.lstsq(A * W[:, None], y * W, rcond=None)
        err = (A @ c - y) / y
        w = w * np.abs(err) + 1e-300
        w /= w.sum()
    c32 = c.astype(np.float32)
    err32 = np.max(np.abs((np.vander(f, deg + 1, increasing=True) @ c32.astype(np.float64) - y) / y))
    return c32, err32


if __name__ == "__main__":
    c, e = fit()
    print("coefficients c0..c3:", ", ".join(f"{float(v):.9g}f" for v in c), f"max rel error {e:.3g}")
