"""Backward (dQ, dK, dV) on the B200 against the oracle and the reference's own
naive backward (golden), over the reference's backward test grid
(tests/test_backward.py:95-105) plus bf16, D=128, causal, GQA and Nk != N.

Tolerance: the reference's backward test uses atol = rtol = 1e-2
(tests/test_backward.py:69-70) for its FP32 kernels; with fp16 inputs and P /
dS rounded to fp16 for the tensor cores that bound holds here too, bf16 (8-bit
mantissa) gets atol = rtol = 5e-2."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from conftest import bits_to_float, golden_files
from oracle import attention as ora

pytestmark = pytest.mark.gpu


def tol(dt):
    return (1e-2, 1e-2) if dt == torch.float16 else (5e-2, 5e-2)


def dev(a, dt):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dt).cuda()


def host(t):
    return t.float().cpu().numpy()


def run_and_check(q, k, v, do, dt, causal=False, what=""):
    import b200attn
    O, L = b200attn.forward(q, k, v, causal=causal)
    dQ, dK, dV = b200attn.backward(q, k, v, O, do, L, causal=causal)
    torch.cuda.synchronize()
    rQ, rK, rV = ora.attention_backward(host(q), host(k), host(v), host(do), causal=causal)
    atol, rtol = tol(dt)
    for name, ours, ref in (("dQ", dQ, rQ), ("dK", dK, rK), ("dV", dV, rV)):
        np.testing.assert_allclose(host(ours), ref, atol=atol, rtol=rtol, err_msg=f"{name} {what}")
    assert b200attn.device_error_flags() == 0


@pytest.mark.parametrize("path", golden_files("backward"), ids=lambda p: os.path.basename(p)[:-4])
def test_golden_backward(path):
    import b200attn
    z = np.load(path)
    name = str(z["dtype"])
    dt = torch.float16 if name == "float16" else torch.bfloat16
    q, k, v, do = (dev(bits_to_float(z[n], name), dt) for n in ("q", "k", "v", "do"))
    O, L = b200attn.forward(q, k, v)
    dQ, dK, dV = b200attn.backward(q, k, v, O, do, L)
    atol, rtol = tol(dt)
    for ours, key in ((dQ, "dQ"), (dK, "dK"), (dV, "dV")):
        np.testing.assert_allclose(host(ours), z[key], atol=atol, rtol=rtol, err_msg=key)


REF_GRID = [(1, 1, 32), (1, 1, 64), (1, 1, 128), (1, 1, 63), (1, 1, 127), (2, 4, 256),
            (2, 8, 512), (1, 1, 1024), (1, 1, 2048)]


@pytest.mark.parametrize("B,H,N", REF_GRID, ids=lambda x: str(x))
def test_reference_backward_grid(B, H, N):
    dt = torch.float16
    q, k, v, do = (dev(ora.seeded_normal((B, H, N, 64), 70 + s), dt) for s in range(4))
    run_and_check(q, k, v, do, dt, False, f"{B},{H},{N}")


VARIANTS = [
    # B, H, Hkv, N, Nk, D, dtype, causal
    (1, 2, 2, 200, 200, 128, torch.bfloat16, False),
    (1, 2, 2, 257, 257, 64, torch.float16, True),
    (1, 4, 4, 300, 300, 128, torch.bfloat16, True),
    (1, 8, 2, 192, 192, 64, torch.float16, False),   # GQA group 4
    (2, 4, 1, 130, 130, 128, torch.float16, True),   # MQA
    (1, 2, 2, 96, 333, 64, torch.float16, True),     # Nk > N, causal aligned to the last key
    (1, 2, 2, 160, 70, 128, torch.bfloat16, False),  # Nk < N
]


@pytest.mark.parametrize("B,H,Hkv,N,Nk,D,dt,causal", VARIANTS, ids=lambda x: str(x))
def test_backward_variants(B, H, Hkv, N, Nk, D, dt, causal):
    q = dev(ora.seeded_normal((B, H, N, D), 90), dt)
    k = dev(ora.seeded_normal((B, Hkv, Nk, D), 91), dt)
    v = dev(ora.seeded_normal((B, Hkv, Nk, D), 92), dt)
    do = dev(ora.seeded_normal((B, H, N, D), 93), dt)
    run_and_check(q, k, v, do, dt, causal, f"{B},{H},{Hkv},{N},{Nk},{D},{causal}")
