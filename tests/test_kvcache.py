"""Paged KV cache: the page allocator (CPU) and append -> paged decode on the GPU."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_parity
from oracle import attention as ora


def test_page_pool_bookkeeping_cpu():
    from b200attn.kvcache import PagePool
    pool = PagePool(num_pages=10, page_size=16, num_kv_heads=2, head_dim=64, max_seqs=3,
                    max_pages=8, device="cpu")
    pool.reserve(0, 17)            # 2 pages
    pool.reserve(1, 16)            # 1 page
    assert pool.num_free == 7
    bt = pool.block_table.numpy()
    assert (bt[0, :2] >= 0).all() and bt[0, 2] == -1 and bt[1, 0] >= 0
    assert len(set(bt[0, :2]) | {bt[1, 0]}) == 3    # no page shared
    with pytest.raises(RuntimeError, match="max_pages"):
        pool.reserve(2, 16 * 9)
    with pytest.raises(RuntimeError, match="exhausted"):
        pool.reserve(2, 16 * 8)
    assert pool.num_free == 7      # the failed reservation was rolled back
    pool.release(0)
    assert pool.num_free == 9 and (pool.block_table.numpy()[0] == -1).all()


@pytest.mark.gpu
def test_append_then_paged_decode_matches_contiguous():
    import b200attn
    from b200attn.kvcache import PagePool
    B, H, Hkv, D, page = 3, 8, 2, 128, 16
    pool = PagePool(num_pages=64, page_size=page, num_kv_heads=Hkv, head_dim=D, max_seqs=B,
                    max_pages=32)
    # a prefill chunk of 40 tokens for every sequence, then 5 single-token decode steps
    chunks = [40, 1, 1, 1, 1, 1]
    K = [ora.seeded_normal((B, Hkv, T, D), 60 + i) for i, T in enumerate(chunks)]
    V = [ora.seeded_normal((B, Hkv, T, D), 80 + i) for i, T in enumerate(chunks)]
    for k, v in zip(K, V):
        pool.append(torch.from_numpy(k).half().cuda(), torch.from_numpy(v).half().cuda())
    torch.cuda.synchronize()
    assert pool.kv_lens.tolist() == [45] * B and pool.lengths() == [45] * B
    q = torch.from_numpy(ora.seeded_normal((B, H, D), 99)).half().cuda()
    O, L = b200attn.decode_paged(q, pool.k_pool, pool.v_pool, pool.block_table, pool.kv_lens,
                                 pages_per_split=4)
    kc = np.concatenate(K, axis=2).astype(np.float16).astype(np.float32)
    vc = np.concatenate(V, axis=2).astype(np.float16).astype(np.float32)
    Or, Lr = ora.decode(q.float().cpu().numpy(), kc, vc)
    assert_parity(O, L, Or, Lr, "float16")
    assert b200attn.device_error_flags() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("D,dt,page", [(128, torch.float16, 16), (64, torch.bfloat16, 32)])
def test_append_is_bit_exact(D, dt, page):
    """The append kernel moves bytes: after a chunk and single-token steps, every
    written pool slot holds exactly the appended K/V bits, and slots past each
    sequence's length are untouched (still zero)."""
    from b200attn.kvcache import PagePool
    B, Hkv = 3, 2
    pool = PagePool(num_pages=40, page_size=page, num_kv_heads=Hkv, head_dim=D, max_seqs=B,
                    max_pages=16, dtype=dt)
    chunks = [37, 1, 1, page]
    K = [torch.from_numpy(ora.seeded_normal((B, Hkv, T, D), 160 + i)).to(dt)
         for i, T in enumerate(chunks)]
    V = [torch.from_numpy(ora.seeded_normal((B, Hkv, T, D), 180 + i)).to(dt)
         for i, T in enumerate(chunks)]
    for k, v in zip(K, V):
        pool.append(k.cuda(), v.cuda())
    torch.cuda.synchronize()
    n = sum(chunks)
    assert pool.lengths() == [n] * B
    kc = torch.cat(K, dim=2).view(torch.int16).numpy()      # [B, Hkv, n, D] raw bits
    vc = torch.cat(V, dim=2).view(torch.int16).numpy()
    kp = pool.k_pool.cpu().view(torch.int16).numpy()        # [P, Hkv, page, D]
    vp = pool.v_pool.cpu().view(torch.int16).numpy()
    bt = pool.block_table.cpu().numpy()
    written = np.zeros(kp.shape[:1] + kp.shape[2:3], dtype=bool)   # [P, page]
    for b in range(B):
        for t in range(n):
            pg, sl = bt[b, t // page], t % page
            assert np.array_equal(kp[pg, :, sl], kc[b, :, t]), (b, t)
            assert np.array_equal(vp[pg, :, sl], vc[b, :, t]), (b, t)
            written[pg, sl] = True
    for pg, sl in zip(*np.nonzero(~written)):
        assert not kp[pg, :, sl].any() and not vp[pg, :, sl].any()
    import b200attn
    assert b200attn.device_error_flags() == 0


@pytest.mark.gpu
def test_append_with_bad_length_is_flagged_not_written():
    """A negative kv_len has no page: the tokens are dropped and bit 2 of the
    device error word is set (nothing is written out of bounds)."""
    import b200attn
    from b200attn.kvcache import append_paged
    B, Hkv, D, page = 2, 1, 64, 16
    kp = torch.zeros(4, Hkv, page, D, dtype=torch.float16, device="cuda")
    vp = torch.zeros_like(kp)
    bt = torch.tensor([[0, 1], [2, 3]], dtype=torch.int32, device="cuda")
    kl = torch.tensor([-5, 0], dtype=torch.int32, device="cuda")
    kn = torch.ones(B, Hkv, 3, D, dtype=torch.float16, device="cuda")
    b200attn.device_error_flags()
    append_paged(kn, kn, kp, vp, bt, kl, advance=False)
    torch.cuda.synchronize()
    assert b200attn.device_error_flags() & 4
    assert not kp[0].any() and not kp[1].any()        # sequence 0 wrote nothing
    assert kp[2, :, :3].eq(1).all()                    # sequence 1 wrote its 3 tokens
