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
