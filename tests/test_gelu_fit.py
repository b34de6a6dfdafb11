"""The epilogues' erf-GELU polynomial (csrc/gemm.cuh gelu_erf, used by the
fused MLP and the GEMM epilogue): the committed coefficients are the fit that
tests/fit_gelu.py produces, and the float32 evaluation stays within 1e-6 of the
exact GELU that the reference's MLP applies (F.gelu,
packages/shrimp/python/shrimp/model.py:513)."""

import importlib.util
import re
from pathlib import Path

import numpy as np

CSRC = Path(__file__).resolve().parents[1] / "hexo_bot_b200" / "csrc"


def _fit_module():
    spec = importlib.util.spec_from_file_location("fit_gelu", Path(__file__).resolve().parent / "fit_gelu.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _kernel_coefficients() -> np.ndarray:
    src = (CSRC / "gemm.cuh").read_text()
    body = src[src.index("float gelu_erf(float x)"):]
    body = body[body.index("float p = "): body.index("asm(")]
    vals = re.findall(r"([-+]?\d\.\d+e[-+]\d+)f", body)
    return np.array([float(v) for v in vals])


def test_kernel_coefficients_match_the_fit():
    fit = _fit_module()
    c = _kernel_coefficients()
    assert c.shape == (fit.DEGREE + 1,)
    np.testing.assert_allclose(c, fit.fit(), rtol=1e-8, atol=1e-12)


def test_float32_gelu_error_below_1e6():
    fit = _fit_module()
    assert fit.max_error(_kernel_coefficients()) < 1e-6
