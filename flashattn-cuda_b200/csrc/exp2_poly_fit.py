"""Fit of the degree-4 polynomial behind exp2_poly2 (sm100_ptx.cuh).

The kernels compute part of their softmax exponentials 2^x on the FMA pipe:
x = n + f with n = round(x) and f in [-1/2, 1/2], 2^f by a polynomial p(f),
2^n by an add to the exponent field.  This script fits p of degree 4 to 2^f
on [-1/2, 1/2] in RELATIVE error: weighted least squares on Chebyshev nodes,
with the weights iteratively raised where the error is largest (Lawson's
method), which converges toward the equiripple (minimax) polynomial.  The
coefficients are then rounded to float32, the precision the kernel uses.

    python exp2_poly_fit.py          # prints the coefficients and the bound

The kernels' coefficients came from this fit; tests/test_exp2_poly.py checks
them against it and checks the whole float32 routine against np.exp2.
"""
from __future__ import annotations

import numpy as np

DEGREE = 4
HALF_WIDTH = 0.5


def fit(degree: int = DEGREE, nodes: int = 2000, iters: int = 400) -> np.ndarray:
    """Coefficients c[0..degree] (c[0] the constant term) of the near-minimax
    relative-error fit of 2^f on [-1/2, 1/2], float64."""
    k = np.arange(nodes)
    f = HALF_WIDTH * np.cos(np.pi * (k + 0.5) / nodes)       # Chebyshev nodes
    y = np.exp2(f)
    A = np.vander(f, degree + 1, increasing=True) / y[:, None]  # relative-error rows
    b = np.ones_like(f)
    w = np.full(nodes, 1.0 / nodes)
    c = None
    for _ in range(iters):
        sw = np.sqrt(w)
        c, *_ = np.linalg.lstsq(A * sw[:, None], b * sw, rcond=None)
        err = np.abs(A @ c - b)
        w = w * err
        w /= w.sum()
    return c


def max_rel_error(c, n: int = 200001) -> float:
    f = np.linspace(-HALF_WIDTH, HALF_WIDTH, n)
    p = np.polyval(np.asarray(c, np.float64)[::-1], f)
    return float(np.max(np.abs(p / np.exp2(f) - 1.0)))


if __name__ == "__main__":
    c = fit()
    c32 = c.astype(np.float32)
    print("coefficients (constant term first), float32:")
    for i, v in enumerate(c32):
        print(f"  c{i} = {float(v)!r}")
    print(f"max relative error: float64 {max_rel_error(c):.3e}, "
          f"float32-rounded {max_rel_error(c32):.3e}")
