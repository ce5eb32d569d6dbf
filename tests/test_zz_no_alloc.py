"""The allocation-free paged decode entry point, b2a_decode_paged_noalloc.

It serves callers that cannot call cudaMalloc where they decode (a runtime
that reserves all device memory up front, a pool that must not grow, a host
that forbids allocation on its request path): the split partials live in a
fixed 16 MiB array inside the library instead of a caller buffer.  This file
is collected last so that a run stopping at the first failure has already run
every other test; it also passes alone in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_parity
from oracle import attention as ora

pytestmark = pytest.mark.gpu


def _paged_case(seed, B, Hkv, D, page, lens, dt):
    rng = np.random.default_rng(seed)
    npages = -(-np.asarray(lens) // page)
    P = int(npages.sum()) + 2
    perm = rng.permutation(P).astype(np.int32)
    bt = np.zeros((B, int(npages.max())), dtype=np.int32)
    pos = 0
    for b in range(B):
        bt[b, :npages[b]] = perm[pos:pos + npages[b]]
        pos += npages[b]
    kp = torch.from_numpy(ora.seeded_normal((P, Hkv, page, D), seed + 1)).to(dt).cuda()
    vp = torch.from_numpy(ora.seeded_normal((P, Hkv, page, D), seed + 2)).to(dt).cuda()
    return kp, vp, torch.from_numpy(bt).cuda(), torch.tensor(lens, dtype=torch.int32).cuda()


def _noalloc(lib, q, kp, vp, bt, kl, pps, dt):
    B, H, D = q.shape
    O = torch.empty((B, H, D), dtype=dt, device="cuda")
    L = torch.empty((B, H), dtype=torch.float32, device="cuda")
    rc = lib.b2a_decode_paged_noalloc(
        q.data_ptr(), kp.data_ptr(), vp.data_ptr(), bt.data_ptr(), kl.data_ptr(),
        O.data_ptr(), L.data_ptr(), B, H, kp.shape[1], D, kp.shape[2], bt.shape[1],
        kp.shape[0], pps, 0 if dt == torch.float16 else 1, D ** -0.5,
        torch.cuda.current_stream().cuda_stream)
    return rc, O, L


def test_noalloc_matches_allocating_entry_point_twice():
    import b200attn
    from b200attn import _lib
    lib = _lib.load()
    cases = [  # two calls in a row, different shapes and contents
        (31, 4, 32, 8, 128, 16, [1, 300, 2000, 17], 8, torch.float16),
        (47, 3, 16, 4, 64, 32, [999, 64, 5], 4, torch.bfloat16),
    ]
    for seed, B, H, Hkv, D, page, lens, pps, dt in cases:
        kp, vp, bt, kl = _paged_case(seed, B, Hkv, D, page, lens, dt)
        q = torch.from_numpy(ora.seeded_normal((B, H, D), seed + 5)).to(dt).cuda()
        rc, O, L = _noalloc(lib, q, kp, vp, bt, kl, pps, dt)
        assert rc == 0, lib.b2a_last_error()
        Oref, Lref = b200attn.decode_paged(q, kp, vp, bt, kl, pages_per_split=pps)
        torch.cuda.synchronize()
        name = "float16" if dt == torch.float16 else "bfloat16"
        assert_parity(O, L, Oref.float().cpu().numpy(), Lref.cpu().numpy(), name, 1.0,
                      f"noalloc vs decode_paged {lens}")
    assert b200attn.device_error_flags() == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from b200attn import _lib
    lib = _lib.load()
    dt = torch.float16
    # 128 * 32 * 64 splits * 129 floats > 4 Mi floats
    q = torch.zeros((128, 32, 128), dtype=dt, device="cuda")
    kp = torch.zeros((4, 8, 16, 128), dtype=dt, device="cuda")
    bt = torch.zeros((128, 64), dtype=torch.int32, device="cuda")
    kl = torch.ones(128, dtype=torch.int32, device="cuda")
    rc, _, _ = _noalloc(lib, q, kp, kp, bt, kl, 1, dt)
    assert rc == 1
    assert b"exceeds the fixed scratch" in lib.b2a_last_error()
