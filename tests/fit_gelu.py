"""Fit of the polynomial used by gelu_erf() in gemm.cuh.

The GEMM epilogue evaluates the exact (erf) GELU as

    GELU(x) = x * Phi(x),  Phi(x) = 1 - 0.5 * exp(-z^2) * R(z)   (x >= 0)
                           Phi(x) =     0.5 * exp(-z^2) * R(z)   (x < 0)
    z = min(|x| / sqrt(2), 4)

where R(z) approximates exp(z^2) * erfc(z), a smooth decreasing function on
[0, 4] that a polynomial fits without the cancellation a fit of erf itself
suffers in float32. R is a degree-11 least-squares fit at 6000 Chebyshev nodes
of [0, 4]; evaluated in float32 (Horner, exp by exp2) the GELU differs from
0.5 * x * (1 + erf(x / sqrt(2))) by at most ~8e-7 for every float32 x.

    python tests/fit_gelu.py     # prints the coefficients and the error
"""

from math import erf, erfc, sqrt

import numpy as np

DEGREE = 11
ZMAX = 4.0


def fit() -> np.ndarray:
    z = (np.cos(np.linspace(0.0, np.pi, 6000)) * 0.5 + 0.5) * ZMAX
    f = np.exp(z * z) * np.vectorize(erfc)(z)
    return np.polyfit(z, f, DEGREE)  # highest power first


def gelu_f32(x: np.ndarray, c: np.ndarray) -> np.ndarray:
    """The epilogue's evaluation, step for step, in float32."""
    x = x.astype(np.float32)
    c = c.astype(np.float32)
    za = np.minimum(np.abs(x) * np.float32(1.0 / sqrt(2.0)), np.float32(ZMAX)).astype(np.float32)
    p = np.full_like(za, c[0])
    for ci in c[1:]:
        p = (p * za + ci).astype(np.float32)
    e = np.exp2((za * (za * np.float32(-1.4426950408889634))).astype(np.float32)).astype(np.float32)
    h = (np.float32(0.5) * p * e).astype(np.float32)
    phi = np.where(x >= 0, np.float32(1.0) - h, h).astype(np.float32)
    return (x * phi).astype(np.float32)


def max_error(c: np.ndarray) -> float:
    xs = np.linspace(-10.0, 10.0, 400001)
    ref = 0.5 * xs * (1.0 + np.vectorize(erf)(xs / sqrt(2.0)))
    return float(np.abs(gelu_f32(xs, c) - ref).max())


if __name__ == "__main__":
    c = fit()
    print("coefficients (highest power first):")
    print(",\n".join(f"  {v:.9e}f" for v in c))
    print(f"max |GELU error| on [-10, 10]: {max_error(c):.2e}")
