"""Variable-length (packed, cu_seqlens) prefill on the B200: parity with the
oracle over ragged batches, empty sequences, sequences with no keys, causal
offsets below zero, GQA, D = 64 / 128 and fp16 / bf16; equality with the
dense forward when all lengths match.  The reference has no varlen form (it
requires K and V to have Q's shape, cuda/flash_attn_fa3_db_full.cu:358-359);
its per-sequence arithmetic is ref/naive_attn.py:27-36."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_parity
from oracle import attention as ora

pytestmark = pytest.mark.gpu

TDT = {"float16": torch.float16, "bfloat16": torch.bfloat16}


@pytest.fixture(scope="module")
def b2a():
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    import b200attn
    return b200attn


def packed(lens_q, lens_k, H, Hkv, D, dtype, seed, amp=1.0):
    cu_q = np.concatenate([[0], np.cumsum(lens_q)]).astype(np.int32)
    cu_k = np.concatenate([[0], np.cumsum(lens_k)]).astype(np.int32)
    tq, tk = int(cu_q[-1]), int(cu_k[-1])
    q = torch.from_numpy(ora.seeded_normal((tq, H, D), seed, amp)).to(dtype).cuda()
    k = torch.from_numpy(ora.seeded_normal((tk, Hkv, D), seed + 1, amp)).to(dtype).cuda()
    v = torch.from_numpy(ora.seeded_normal((tk, Hkv, D), seed + 2, amp)).to(dtype).cuda()
    return q, k, v, cu_q, cu_k


def run_case(b2a, lens_q, lens_k, H, Hkv, D, dt, causal, seed=0):
    dtype = TDT[dt]
    q, k, v, cu_q, cu_k = packed(lens_q, lens_k, H, Hkv, D, dtype, seed)
    O, L = b2a.forward_varlen(q, k, v, torch.from_numpy(cu_q).cuda(),
                              torch.from_numpy(cu_k).cuda(), max(lens_q), causal=causal)
    torch.cuda.synchronize()
    assert b2a.device_error_flags() == 0
    O_ref, L_ref = ora.varlen_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                        v.float().cpu().numpy(), cu_q, cu_k, causal=causal)
    assert O.shape == q.shape and L.shape == (H, q.shape[0])
    assert_parity(O, L, O_ref, L_ref, dt, 1.0, f"varlen {lens_q} {lens_k} causal={causal}")
    return O, L


CASES = [
    # lens_q, lens_k
    ([1, 127, 128, 129, 300], [1, 127, 128, 129, 300]),      # self-attention, ragged
    ([256, 1, 513], [700, 5, 513]),                           # Nk > N (chunk over a cache)
    ([64, 0, 200], [64, 90, 200]),                            # an empty query sequence
]


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dt", ["float16", "bfloat16"])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_varlen_parity(b2a, D, dt, causal, case):
    lens_q, lens_k = CASES[case]
    run_case(b2a, lens_q, lens_k, 4, 2, D, dt, causal, seed=10 + case)


@pytest.mark.parametrize("causal", [False, True])
def test_varlen_rows_without_keys(b2a, causal):
    # sequence 1 has no keys; with causal, sequence 2 (N=300 > Nk=100) has
    # 200 rows that see no key: O = 0, L = -inf there
    O, L = run_case(b2a, [50, 40, 300], [60, 0, 100], 2, 2, 128, "bfloat16", causal, seed=3)
    assert torch.all(O[50:90] == 0) and torch.all(torch.isinf(L[:, 50:90]))
    if causal:
        assert torch.all(O[90:290] == 0) and torch.all(L[:, 90:290] == -float("inf"))


def test_varlen_matches_dense(b2a):
    # equal lengths: the packed layout over the same kernel must give the dense
    # forward's bits (D = 128 runs the same kernel in both layouts)
    B, H, N, D = 3, 4, 384, 128
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    for causal in (False, True):
        O, L = b2a.forward(q, k, v, causal=causal)
        cu = torch.arange(0, (B + 1) * N, N, dtype=torch.int32, device="cuda")
        pk = lambda t: t.permute(0, 2, 1, 3).reshape(B * N, H, D)
        Ov, Lv = b2a.forward_varlen(pk(q), pk(k), pk(v), cu, cu, N, causal=causal)
        assert torch.equal(Ov, pk(O))
        assert torch.equal(Lv, L.permute(1, 0, 2).reshape(H, B * N))


def test_varlen_long_and_gqa(b2a):
    run_case(b2a, [2048, 1000], [2048, 3000], 8, 2, 128, "float16", True, seed=7)


def test_varlen_max_seqlen_too_small_flags(b2a):
    dtype = torch.float16
    q, k, v, cu_q, cu_k = packed([600], [600], 1, 1, 64, dtype, 1)
    b2a.device_error_flags()
    b2a.forward_varlen(q, k, v, torch.from_numpy(cu_q).cuda(), torch.from_numpy(cu_k).cuda(), 256)
    torch.cuda.synchronize()
    assert b2a.device_error_flags() & 8


def test_varlen_errors(b2a):
    q = torch.zeros(10, 4, 128, dtype=torch.float16, device="cuda")
    cu = torch.tensor([0, 10], dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="must be int32"):
        b2a.forward_varlen(q, q, q, cu.long(), cu.long(), 10)
    with pytest.raises(RuntimeError, match="Head dimension"):
        b2a.forward_varlen(q[..., :32], q[..., :32], q[..., :32], cu, cu, 10)
    with pytest.raises(RuntimeError, match="max_seqlen_q"):
        b2a.forward_varlen(q, q, q, cu, cu, 11)
