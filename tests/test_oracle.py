"""The CPU oracle, pinned against golden vectors produced by the reference's own
ref/naive_attn.py (tests/golden/make_golden.py), plus the algebraic identities
the decode restatements rely on.  CPU only."""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import golden_files, load_golden
from oracle import attention as ora

PREFILL = golden_files("prefill")
DECODE = golden_files("decode")


def test_fixture_inventory():
    # the reference grid (tests/test_fa3_db_full.py:58-75) + extensions
    names = {os.path.basename(p) for p in PREFILL + DECODE}
    for n in (1, 2, 7, 31, 33, 63, 64, 127, 128):
        assert f"prefill_n{n}.npz" in names
    assert len(PREFILL) >= 15 and len(DECODE) >= 3


@pytest.mark.parametrize("path", PREFILL, ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_matches_reference_prefill(path):
    g = load_golden(path)
    O, L = ora.naive_attention(g["q"], g["k"], g["v"])
    # golden is the reference evaluated in fp32; the oracle runs in fp64
    # fp32 rounding of the reference grows with the logit scale (amp^2)
    np.testing.assert_allclose(O, g["O"], atol=2e-5 * max(g["amp"], 1.0) ** 2, rtol=1e-4)
    np.testing.assert_allclose(L, g["L"], atol=1e-5 * max(g["amp"], 1.0) ** 2, rtol=1e-5)


@pytest.mark.parametrize("path", DECODE, ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_matches_reference_decode(path):
    g = load_golden(path)
    O, L = ora.decode(g["q"][:, :, 0], g["k"], g["v"])
    np.testing.assert_allclose(O, g["O"][:, :, 0], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(L, g["L"][:, :, 0], atol=1e-5, rtol=1e-5)


def test_oracle_fp32_mode_tracks_reference_bits():
    g = load_golden(PREFILL[0])
    O, L = ora.naive_attention(g["q"], g["k"], g["v"], dtype=np.float32)
    np.testing.assert_allclose(O, g["O"], atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("splits", [1, 3, 7, 16, 40])
def test_split_partials_combine_to_full(splits):
    q = ora.seeded_normal((2, 8, 64), 1)
    k = ora.seeded_normal((2, 2, 33, 64), 2)
    v = ora.seeded_normal((2, 2, 33, 64), 3)
    O, L = ora.decode(q, k, v)
    op, lp = ora.decode_splitkv_partials(q, k, v, splits)
    if splits > 33:
        assert np.isneginf(lp[..., -1]).all()
    O2, L2 = ora.combine(op, lp)
    np.testing.assert_allclose(O2, O, atol=1e-12, rtol=1e-10)
    np.testing.assert_allclose(L2, L, atol=1e-12, rtol=1e-10)


def test_gqa_equals_repeated_heads():
    q = ora.seeded_normal((1, 8, 20, 64), 4)
    k = ora.seeded_normal((1, 2, 20, 64), 5)
    v = ora.seeded_normal((1, 2, 20, 64), 6)
    O, L = ora.naive_attention(q, k, v)
    O2, L2 = ora.naive_attention(q, np.repeat(k, 4, axis=1), np.repeat(v, 4, axis=1))
    np.testing.assert_array_equal(O, O2)
    np.testing.assert_array_equal(L, L2)


def test_causal_row_equals_prefix_attention():
    q = ora.seeded_normal((1, 1, 40, 64), 7)
    k = ora.seeded_normal((1, 1, 40, 64), 8)
    v = ora.seeded_normal((1, 1, 40, 64), 9)
    O, L = ora.naive_attention(q, k, v, causal=True)
    for r in (0, 1, 17, 39):
        o, l = ora.attention_head(q[0, 0, r:r + 1], k[0, 0, :r + 1], v[0, 0, :r + 1], 64 ** -0.5)
        np.testing.assert_allclose(O[0, 0, r], o[0], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(L[0, 0, r], l[0], rtol=1e-12)
    Or, Lr = ora.attention_rows(q, k, v, 0, 0, [5, 30], causal=True)
    np.testing.assert_allclose(Or, O[0, 0, [5, 30]], rtol=1e-12, atol=1e-12)


def test_paged_gather_equals_contiguous():
    rng = np.random.default_rng(0)
    B, Hkv, D, page = 3, 2, 64, 16
    lens = np.array([1, 40, 77])
    npages = -(-lens // page)
    P = int(npages.sum()) + 2
    perm = rng.permutation(P)
    bt = np.zeros((B, int(npages.max())), dtype=np.int32)
    pos = 0
    for b in range(B):
        bt[b, :npages[b]] = perm[pos:pos + npages[b]]
        pos += npages[b]
    kp = ora.seeded_normal((P, Hkv, page, D), 10)
    vp = ora.seeded_normal((P, Hkv, page, D), 11)
    q = ora.seeded_normal((B, 4, D), 12)
    O, L = ora.decode_paged(q, kp, vp, bt, lens)
    for b in range(B):
        kc = ora.paged_gather(kp, bt[b], lens[b])
        assert kc.shape == (Hkv, lens[b], D)
        o, l = ora.decode(q[b:b + 1], kc[None], ora.paged_gather(vp, bt[b], lens[b])[None])
        np.testing.assert_allclose(O[b], o[0], rtol=1e-12, atol=1e-12)


def test_causal_cross_mask_aligned_to_last_key():
    q = ora.seeded_normal((1, 1, 5, 16), 20)
    k = ora.seeded_normal((1, 1, 9, 16), 21)
    v = ora.seeded_normal((1, 1, 9, 16), 22)
    O, L = ora.naive_attention(q, k, v, causal=True)
    for r in range(5):  # row r sees keys 0 .. r + 4
        o, l = ora.attention_head(q[0, 0, r:r + 1], k[0, 0, :r + 5], v[0, 0, :r + 5], 0.25)
        np.testing.assert_allclose(O[0, 0, r], o[0], rtol=1e-12, atol=1e-12)


BACKWARD = golden_files("backward")


@pytest.mark.parametrize("path", BACKWARD, ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_backward_matches_reference(path):
    from conftest import bits_to_float
    z = np.load(path)
    dt = str(z["dtype"])
    q, k, v, do = (bits_to_float(z[n], dt) for n in ("q", "k", "v", "do"))
    dQ, dK, dV = ora.attention_backward(q, k, v, do)
    for ours, ref in ((dQ, z["dQ"]), (dK, z["dK"]), (dV, z["dV"])):
        np.testing.assert_allclose(ours, ref, atol=1e-4, rtol=1e-4)


def test_oracle_backward_matches_finite_differences():
    q = ora.seeded_normal((1, 2, 6, 8), 30).astype(np.float64)
    k = ora.seeded_normal((1, 1, 9, 8), 31).astype(np.float64)
    v = ora.seeded_normal((1, 1, 9, 8), 32).astype(np.float64)
    do = ora.seeded_normal((1, 2, 6, 8), 33).astype(np.float64)
    dQ, dK, dV = ora.attention_backward(q, k, v, do, causal=True)
    f = lambda q_, k_, v_: (ora.naive_attention(q_, k_, v_, causal=True)[0] * do).sum()
    eps = 1e-6
    for arr, grad in ((q, dQ), (k, dK), (v, dV)):
        idx = (0, 0, 3, 5)
        a1, a2 = arr.copy(), arr.copy()
        a1[idx] += eps
        a2[idx] -= eps
        args1 = [a1 if arr is x else x for x in (q, k, v)]
        args2 = [a2 if arr is x else x for x in (q, k, v)]
        num = (f(*args1) - f(*args2)) / (2 * eps)
        np.testing.assert_allclose(grad[idx], num, rtol=1e-6, atol=1e-8)


@pytest.mark.parametrize("causal", [False, True])
def test_varlen_oracle_matches_dense(causal):
    """Packed varlen with equal lengths is the dense computation re-laid out."""
    B, H, Hkv, N, Nk, D = 2, 4, 2, 37, 53, 16
    Q = ora.seeded_normal((B, H, N, D), 1)
    K = ora.seeded_normal((B, Hkv, Nk, D), 2)
    V = ora.seeded_normal((B, Hkv, Nk, D), 3)
    O, L = ora.naive_attention(Q, K, V, causal=causal)
    pk = lambda t: t.transpose(0, 2, 1, 3).reshape(-1, t.shape[1], D)
    cu_q = np.arange(0, (B + 1) * N, N)
    cu_k = np.arange(0, (B + 1) * Nk, Nk)
    Ov, Lv = ora.varlen_attention(pk(Q), pk(K), pk(V), cu_q, cu_k, causal=causal)
    np.testing.assert_allclose(Ov, pk(O), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(Lv, L.transpose(1, 0, 2).reshape(H, -1), rtol=1e-12)
