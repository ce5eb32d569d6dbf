"""CPU oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this module, and only as the checker or the timed CPU
baseline.  The product path (b200attn) never calls it and has no CPU fallback.

Every function restates, in numpy, the reference's naive attention
(ref/naive_attn.py:10-38):

    S = Q K^T * D^-0.5;  P = softmax(S);  O = P V;  L = logsumexp(S)

with the extensions the B200 library adds (causal mask, GQA head sharing,
explicit scale, decode with query length 1, split-KV partials and their
LSE-weighted combine, paged-KV gather).  Arithmetic is float64 by default so
that the oracle's own rounding is far below the tolerances under test; pass
dtype=np.float32 to reproduce the reference's fp32 evaluation.

Pinning: tests/test_oracle.py checks this module against golden vectors that
tests/golden/make_golden.py produced by running the reference's own
ref/naive_attn.py (torch, CPU) on seeded inputs, and against the reference
tests' shape grid (tests/test_fa3_db_full.py:58-75).
"""
from __future__ import annotations

import numpy as np


def _kv_head(h: int, H: int, Hkv: int) -> int:
    """Query head h reads KV head h // (H / Hkv) (GQA; identity when Hkv == H)."""
    return h // (H // Hkv)


def attention_head(q, k, v, scale, causal=False, row_offset=0, dtype=np.float64):
    """One head: q [M, D] (query rows row_offset..row_offset+M-1), k/v [N, D].

    Returns (O [M, D], L [M]).  Restates ref/naive_attn.py:27-36 for one
    (b, h) slice; the causal mask keeps key j <= query row i.
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    s = (q @ k.T) * dtype(scale)                     # S = Q K^T * scale   (:27)
    if causal:
        rows = np.arange(q.shape[0])[:, None] + row_offset
        cols = np.arange(k.shape[0])[None, :]
        s = np.where(cols <= rows, s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    z = e.sum(axis=-1, keepdims=True)
    p = e / z                                        # P = softmax(S)      (:30)
    o = p @ v                                        # O = P V             (:33)
    lse = (m + np.log(z))[:, 0]                      # L = logsumexp(S)    (:36)
    return o, lse


def naive_attention(Q, K, V, scale=None, causal=False, dtype=np.float64):
    """Q [B,H,N,D], K/V [B,Hkv,Nk,D] -> (O [B,H,N,D], L [B,H,N]) (ref/naive_attn.py:10-38).

    With Nk != N the causal mask is aligned to the last key: row r sees keys
    0 .. r + Nk - N (the reference only has Nk == N)."""
    Q = np.asarray(Q)
    B, H, N, D = Q.shape
    Hkv = K.shape[1]
    scale = D ** -0.5 if scale is None else scale
    O = np.empty((B, H, N, D), dtype=dtype)
    L = np.empty((B, H, N), dtype=dtype)
    for b in range(B):
        for h in range(H):
            hk = _kv_head(h, H, Hkv)
            O[b, h], L[b, h] = attention_head(Q[b, h], K[b, hk], V[b, hk], scale, causal,
                                              K.shape[2] - N, dtype)
    return O, L


def varlen_attention(Q, K, V, cu_q, cu_k, scale=None, causal=False, dtype=np.float64):
    """Packed variable-length attention: Q [total_q,H,D], K/V [total_k,Hkv,D].

    Sequence b is query tokens cu_q[b]..cu_q[b+1]-1 over keys
    cu_k[b]..cu_k[b+1]-1, each computed as naive_attention of that one
    sequence (the reference's per-(b, h) computation, ref/naive_attn.py:27-36).
    Returns (O [total_q,H,D], L [H,total_q]).  Causal masks align per sequence
    to its last key; a row that sees no key gets O = 0 and L = -inf.
    """
    Q = np.asarray(Q)
    total_q, H, D = Q.shape
    Hkv = K.shape[1]
    scale = D ** -0.5 if scale is None else scale
    O = np.zeros((total_q, H, D), dtype=dtype)
    L = np.full((H, total_q), -np.inf, dtype=dtype)
    for b in range(len(cu_q) - 1):
        q0, q1, k0, k1 = int(cu_q[b]), int(cu_q[b + 1]), int(cu_k[b]), int(cu_k[b + 1])
        n, nk = q1 - q0, k1 - k0
        for h in range(H):
            hk = _kv_head(h, H, Hkv)
            for r in range(n):
                last = (r + nk - n) if causal else nk - 1  # last visible key
                if last < 0:
                    continue
                o, l = attention_head(Q[q0 + r, h][None], K[k0:k0 + last + 1, hk],
                                      V[k0:k0 + last + 1, hk], scale, False, 0, dtype)
                O[q0 + r, h], L[h, q0 + r] = o[0], l[0]
    return O, L


def attention_rows(Q, K, V, b, h, rows, scale=None, causal=False, dtype=np.float64):
    """O and L of selected query rows of head (b, h): for spot checks at large N."""
    B, H, N, D = Q.shape
    Hkv = K.shape[1]
    scale = D ** -0.5 if scale is None else scale
    hk = _kv_head(h, H, Hkv)
    rows = np.asarray(rows)
    outs_o, outs_l = [], []
    for r in rows:
        kk = K[b, hk, : r + 1] if causal else K[b, hk]
        vv = V[b, hk, : r + 1] if causal else V[b, hk]
        o, l = attention_head(Q[b, h, r:r + 1], kk, vv, scale, False, 0, dtype)
        outs_o.append(o[0])
        outs_l.append(l[0])
    return np.stack(outs_o), np.array(outs_l)


# ------------------------------------------------------------------------ decode

def decode(q, k, v, scale=None, dtype=np.float64):
    """q [B,H,D], k/v [B,Hkv,Lkv,D] -> (O [B,H,D], L [B,H]): attention of one query row."""
    B, H, D = q.shape
    Hkv = k.shape[1]
    scale = D ** -0.5 if scale is None else scale
    O = np.empty((B, H, D), dtype=dtype)
    L = np.empty((B, H), dtype=dtype)
    for b in range(B):
        for h in range(H):
            hk = _kv_head(h, H, Hkv)
            o, l = attention_head(q[b, h][None], k[b, hk], v[b, hk], scale, False, 0, dtype)
            O[b, h], L[b, h] = o[0], l[0]
    return O, L


def decode_splitkv_partials(q, k, v, splits, scale=None, dtype=np.float64):
    """Per-split partials: (o_part [B,H,S,D], l_part [B,H,S]).

    Split s covers tokens [s*c, min(Lkv, (s+1)*c)) with c = ceil(Lkv/S); o is the
    softmax-normalised output over the split, l its natural-log sum of exp; an
    empty split has l = -inf and o = 0.
    """
    B, H, D = q.shape
    Hkv, Lkv = k.shape[1], k.shape[2]
    scale = D ** -0.5 if scale is None else scale
    c = -(-Lkv // splits)
    o_part = np.zeros((B, H, splits, D), dtype=dtype)
    l_part = np.full((B, H, splits), -np.inf, dtype=dtype)
    for s in range(splits):
        t0, t1 = s * c, min(Lkv, (s + 1) * c)
        if t0 >= t1:
            continue
        o, l = decode(q, k[:, :, t0:t1], v[:, :, t0:t1], scale, dtype)
        o_part[:, :, s], l_part[:, :, s] = o, l
    return o_part, l_part


def combine(o_part, l_part, dtype=np.float64):
    """L = log sum_s exp(l_s);  O = sum_s exp(l_s - L) o_s  (online-softmax rescale,
    cuda/flash_attn_fa3_db_full.cu:261-284 and :340, applied across splits)."""
    o_part = np.asarray(o_part, dtype=dtype)
    l_part = np.asarray(l_part, dtype=dtype)
    M = l_part.max(axis=-1, keepdims=True)
    w = np.where(np.isneginf(l_part), 0.0, np.exp(l_part - M))
    Z = w.sum(axis=-1, keepdims=True)
    O = (w[..., None] * o_part).sum(axis=-2) / Z
    L = (M + np.log(Z))[..., 0]
    return O, L


def paged_gather(pool, block_table_row, length):
    """Contiguous [Hkv, length, D] view of one sequence from a [P, Hkv, page, D] pool."""
    page = pool.shape[2]
    npages = -(-length // page)
    pages = [pool[block_table_row[i]] for i in range(npages)]      # each [Hkv, page, D]
    return np.concatenate(pages, axis=1)[:, :length]


def decode_paged(q, k_pool, v_pool, block_table, kv_lens, scale=None, dtype=np.float64):
    """Paged decode: token t of sequence b is slot t % page of page block_table[b, t // page]."""
    B, H, D = q.shape
    O = np.empty((B, H, D), dtype=dtype)
    L = np.empty((B, H), dtype=dtype)
    for b in range(B):
        kb = paged_gather(k_pool, block_table[b], int(kv_lens[b]))[None]
        vb = paged_gather(v_pool, block_table[b], int(kv_lens[b]))[None]
        o, l = decode(q[b:b + 1], kb, vb, scale, dtype)
        O[b], L[b] = o[0], l[0]
    return O, L


# ----------------------------------------------------------------- seeded inputs

def seeded_normal(shape, seed, amp=1.0):
    """N(0,1)*amp float32 values from a seeded generator (device-independent bits)."""
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(amp))


# ---------------------------------------------------------------------- backward

def attention_backward(Q, K, V, dO, scale=None, causal=False, dtype=np.float64):
    """(dQ, dK, dV) of O = softmax(Q K^T * scale) V for upstream gradient dO.

    Restates the reference's naive backward (tests/test_backward.py:20-46) and
    the kernels it checks (cuda/flash_attn_kernel.cu:173-412):
        P = softmax(S);  dV = P^T dO;  dP = dO V^T;  D_i = rowsum(dO * O);
        dS = P * (dP - D_i);  dQ = dS K * scale;  dK = dS^T Q * scale
    with the same causal mask (aligned to the last key) and GQA head sharing as
    naive_attention: dK/dV of a KV head sum over the query heads that use it.
    """
    B, H, N, D = Q.shape
    Hkv, Nk = K.shape[1], K.shape[2]
    scale = D ** -0.5 if scale is None else scale
    dQ = np.zeros((B, H, N, D), dtype=dtype)
    dK = np.zeros((B, Hkv, Nk, D), dtype=dtype)
    dV = np.zeros((B, Hkv, Nk, D), dtype=dtype)
    for b in range(B):
        for h in range(H):
            hk = _kv_head(h, H, Hkv)
            q, k, v, do = (np.asarray(x, dtype=dtype) for x in (Q[b, h], K[b, hk], V[b, hk], dO[b, h]))
            s = (q @ k.T) * dtype(scale)
            if causal:
                rows = np.arange(N)[:, None] + (Nk - N)
                s = np.where(np.arange(Nk)[None, :] <= rows, s, -np.inf)
            m = s.max(axis=-1, keepdims=True)
            p = np.exp(s - m)
            p /= p.sum(axis=-1, keepdims=True)
            o = p @ v
            dV[b, hk] += p.T @ do
            dp = do @ v.T
            di = (do * o).sum(axis=-1, keepdims=True)
            ds = p * (dp - di)
            dQ[b, h] = ds @ k * scale
            dK[b, hk] += ds.T @ q * scale
    return dQ, dK, dV
