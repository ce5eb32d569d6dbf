"""Shared test setup: the `gpu` marker, import paths and golden-fixture loading."""
from __future__ import annotations

import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_PARENT = os.path.join(ROOT, "flashattn-cuda_b200")
for p in (ROOT, PKG_PARENT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and libb200attn.so")


def bits_to_float(bits: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values of raw float16 / bfloat16 bit patterns."""
    bits = np.asarray(bits, dtype=np.uint16)
    if dtype == "float16":
        return bits.view(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return (bits.astype(np.uint32) << 16).view(np.float32)
    raise ValueError(dtype)


def load_golden(path: str) -> dict:
    z = np.load(path)
    dt = str(z["dtype"])
    out = {"dtype": dt, "O": z["O"].astype(np.float32), "L": z["L"].astype(np.float32),
           "amp": float(z["amp"]) if "amp" in z.files else 1.0,
           "name": os.path.basename(path)[:-4]}
    for key in ("q", "k", "v"):
        out[key] = bits_to_float(z[key], dt)
    return out


def golden_files(prefix: str) -> list[str]:
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, f"{prefix}_*.npz")))


# ----------------------------------------------------------------- GPU helpers
def parity_tol(dtype: str, amp: float = 1.0):
    """(O atol, O rtol): the reference test's fp16 bound (tests/test_fa3_db_full.py:43,
    atol 2e-3*max(amp,1), rtol 2e-3) and the bf16 bound (atol 1e-2, rtol 2e-2)."""
    if dtype in ("bfloat16", "bf16"):
        return 1e-2 * max(amp, 1.0), 2e-2
    return 2e-3 * max(amp, 1.0), 2e-3


L_RTOL = 1e-4   # L within 1e-4 relative ...
L_ATOL = 1e-5   # ... plus a floor for |L| ~ 0 (N = 1 rows)


def assert_parity(O, L, O_ref, L_ref, dtype: str, amp: float = 1.0, what: str = ""):
    """Compare kernel outputs (torch, any device) with float reference arrays."""
    O = O.float().cpu().numpy()
    atol, rtol = parity_tol(dtype, amp)
    np.testing.assert_allclose(O, np.asarray(O_ref, np.float64), atol=atol, rtol=rtol,
                               err_msg=f"O mismatch {what}")
    if L is not None:
        L = L.float().cpu().numpy()
        np.testing.assert_allclose(L, np.asarray(L_ref, np.float64),
                                   atol=L_ATOL * max(amp, 1.0), rtol=L_RTOL,
                                   err_msg=f"L mismatch {what}")
