"""Fit of the polynomial used by gelu_erf() in gemm.cuh.

The epilogues evaluate the exact (erf) GELU as

    GELU(x) = max(x, 0) - u * q(u) * exp(-u^2 / 2),   u = min(|x|, 4 sqrt(2))

which is x * Phi(x) written through 1 - Phi(|x|) = 0.5 * erfc(|x| / sqrt(2))
= exp(-x^2 / 2) * q(|x|), with q(u) = 0.5 * exp(u^2 / 2) * erfc(u / sqrt(2)) a
smooth decreasing function on [0, 4 sqrt(2)] that a polynomial fits without
the cancellation a fit of erf itself suffers in float32. Past the clamp the
correction term is below 1e-7. In float32 the evaluation is one min, nine
Horner FMAs, two multiplies for the exponent, one exp2, one multiply, one
NaN-propagating max and one FMA.

q is a degree-9 polynomial fitted at 8000 Chebyshev nodes by least squares
weighted with u * exp(-u^2 / 2) (the factor the fit error is multiplied by in
the GELU), re-weighted 30 times toward the nodes with the largest weighted
error (Lawson's iteration toward the minimax fit). Evaluated in float32 the
GELU differs from 0.5 * x * (1 + erf(x / sqrt(2))) by at most ~7e-7 for every
float32 x.

    python tests/fit_gelu.py     # prints the coefficients and the error
"""

from math import erf, erfc, sqrt

import numpy as np

DEGREE = 9
UMAX = 4.0 * sqrt(2.0)
LOG2E = 1.4426950408889634


def fit() -> np.ndarray:
    u = (np.cos(np.linspace(0.0, np.pi, 8000)) * 0.5 + 0.5) * UMAX
    f = 0.5 * np.exp(u * u / 2.0) * np.vectorize(erfc)(u / sqrt(2.0))
    damp = u * np.exp(-u * u / 2.0)
    w = damp + 1e-3
    for _ in range(30):
        c = np.polyfit(u, f, DEGREE, w=w)
        r = np.abs(np.polyval(c, u) - f) * (damp + 1e-9)
        w = w * (1.0 + r / r.max())
    return c  # highest power first


def gelu_f32(x: np.ndarray, c: np.ndarray) -> np.ndarray:
    """The epilogue's evaluation, step for step, in float32."""
    x = x.astype(np.float32)
    c = c.astype(np.float32)
    u = np.minimum(np.abs(x), np.float32(UMAX)).astype(np.float32)
    p = np.full_like(u, c[0])
    for ci in c[1:]:
        p = (p * u + ci).astype(np.float32)
    k = np.float32(-0.5 * LOG2E)
    e = np.exp2((u * (u * k).astype(np.float32)).astype(np.float32)).astype(np.float32)
    t = (u * p).astype(np.float32)
    return (np.maximum(x, np.float32(0.0)) - t * e).astype(np.float32)


def max_error(c: np.ndarray) -> float:
    xs = np.linspace(-12.0, 12.0, 480001)
    ref = 0.5 * xs * (1.0 + np.vectorize(erf)(xs / sqrt(2.0)))
    return float(np.abs(gelu_f32(xs, c) - ref).max())


if __name__ == "__main__":
    c = fit()
    print("coefficients (highest power first):")
    print(",\n".join(f"  {v:.9e}f" for v in c))
    print(f"max |GELU error| on [-12, 12]: {max_error(c):.2e}")
