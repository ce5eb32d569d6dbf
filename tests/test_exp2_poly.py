"""The FMA-pipe exp2 of the softmax (exp2_poly2 in sm100_ptx.cuh), checked on
the CPU: its coefficients against the committed fit
(flashattn-cuda_b200/csrc/exp2_poly_fit.py), and a float32 restatement of the
whole routine -- range reduction, polynomial, exponent add -- against np.exp2
over the softmax's input range [-126, 0] (the kernels only exponentiate
s - max <= 0; a few positive inputs are checked too).  The reference uses
exp2f throughout its softmax (cuda/flash_attn_fa3_db_full.cu:263-272); the
bound here is the fit's 2.6e-6 maximum relative error plus float32 rounding of
the Horner steps."""
from __future__ import annotations

import importlib.util
import os
import re

import numpy as np

from conftest import ROOT

CSRC = os.path.join(ROOT, "flashattn-cuda_b200", "csrc")


def kernel_coefficients() -> np.ndarray:
    """c0..c4 (constant term first) as written in exp2_poly2."""
    text = open(os.path.join(CSRC, "sm100_ptx.cuh")).read()
    body = text[text.index("float2 exp2_poly2"):]
    body = body[:body.index("return p;")]
    vals = [float(v) for v in re.findall(r"make_float2\(([0-9.]+)f,", body)]
    # the Horner chain: first pair (c4, c3), then c2, c1, c0
    c4, c3, c2, c1, c0 = vals[-5:]
    return np.array([c0, c1, c2, c3, c4], dtype=np.float32)


def fit_module():
    spec = importlib.util.spec_from_file_location("exp2_poly_fit",
                                                  os.path.join(CSRC, "exp2_poly_fit.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def fma32(a, b, c):
    """float32 fused multiply-add: the float64 product of two float32 values is
    exact, so one rounding of the float64 sum to float32 models fma.rn.f32 (up to
    a rare double rounding, far below the bound tested)."""
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_poly_f32(x: np.ndarray, c: np.ndarray) -> np.ndarray:
    """float32 restatement of exp2_poly2 (sm100_ptx.cuh)."""
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    shift = np.float32(12582912.0)                 # 1.5 * 2^23
    t = (x + shift).astype(np.float32)             # round(x) in the low mantissa bits
    n = (t - shift).astype(np.float32)
    f = (x - n).astype(np.float32)
    p = fma32(np.full_like(f, c[4]), f, np.full_like(f, c[3]))
    p = fma32(p, f, np.full_like(f, c[2]))
    p = fma32(p, f, np.full_like(f, c[1]))
    p = fma32(p, f, np.full_like(f, c[0]))
    pi = p.view(np.int32) + (t.view(np.int32) << 23)
    return pi.astype(np.int32).view(np.float32)


def test_kernel_coefficients_are_the_fit():
    mod = fit_module()
    c = kernel_coefficients()
    fitted = mod.fit().astype(np.float32)
    np.testing.assert_allclose(c, fitted, rtol=1e-6, atol=0)
    assert mod.max_rel_error(c.astype(np.float64)) < 2.7e-6


def test_exp2_poly_relative_error_over_softmax_range():
    c = kernel_coefficients()
    rng = np.random.default_rng(0)
    x = np.concatenate([np.linspace(-126.0, 0.0, 400001, dtype=np.float32),
                        rng.uniform(-30.0, 0.0, 200000).astype(np.float32),
                        np.arange(-126, 1, dtype=np.float32) + np.float32(0.5),
                        np.array([0.0, -0.5, 0.5, 3.75, 20.25, 63.0], np.float32)])
    y = exp2_poly_f32(x, c).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y / ref - 1.0)
    assert np.all(np.isfinite(y))
    assert rel.max() < 3.0e-6, float(rel.max())


def test_exp2_poly_clamps_below_minus_126():
    c = kernel_coefficients()
    x = np.array([-127.0, -200.0, -1e30, -np.inf], np.float32)
    y = exp2_poly_f32(x, c)
    assert np.all(np.isfinite(y)) and np.all(y > 0) and np.all(y < 2e-38)
