"""Split-KV, combine and paged decode on the B200 against the CPU oracle and the
reference-generated decode golden vectors (query length 1)."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from conftest import assert_parity, golden_files, load_golden
from oracle import attention as ora

pytestmark = pytest.mark.gpu

TDT = {"float16": torch.float16, "bfloat16": torch.bfloat16}
NAME = {torch.float16: "float16", torch.bfloat16: "bfloat16"}


@pytest.fixture(scope="module")
def b2a():
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    import b200attn
    return b200attn


def dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).cuda()


def host(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("splits", [1, 4, 16])
@pytest.mark.parametrize("path", golden_files("decode"), ids=lambda p: os.path.basename(p)[:-4])
def test_golden_decode(b2a, path, splits):
    g = load_golden(path)
    dt = TDT[g["dtype"]]
    q, k, v = dev(g["q"], dt), dev(g["k"], dt), dev(g["v"], dt)   # q [B,H,1,D]
    O, L = b2a.decode(q, k, v, splits=splits)
    assert O.shape == q.shape and L.shape == q.shape[:3]
    assert_parity(O, L, g["O"], g["L"], g["dtype"], 1.0, g["name"])


CASES = [
    # B, H, Hkv, Lkv, D, dtype, splits
    (2, 8, 2, 1000, 128, torch.float16, 4),
    (2, 8, 8, 333, 64, torch.float16, 3),
    (1, 16, 2, 777, 128, torch.bfloat16, 5),
    (3, 4, 2, 64, 64, torch.bfloat16, 1),
    (1, 4, 4, 1, 128, torch.float16, 1),
    (1, 8, 1, 100, 128, torch.float16, 7),
    (2, 4, 1, 40, 64, torch.float16, 64),     # more splits than tokens: empty splits
    (1, 32, 8, 4096, 128, torch.float16, 16),
]


@pytest.mark.parametrize("B,H,Hkv,Lkv,D,dt,splits", CASES, ids=lambda x: str(x))
def test_splitkv_partials_and_combine(b2a, B, H, Hkv, Lkv, D, dt, splits):
    q = dev(ora.seeded_normal((B, H, D), 1), dt)
    k = dev(ora.seeded_normal((B, Hkv, Lkv, D), 2), dt)
    v = dev(ora.seeded_normal((B, Hkv, Lkv, D), 3), dt)
    op, lp = b2a.decode_splitkv(q, k, v, splits=splits)
    opr, lpr = ora.decode_splitkv_partials(host(q), host(k), host(v), splits)
    empty = np.isneginf(lpr)
    assert (np.isneginf(host(lp)) == empty).all()
    atol, rtol = (2e-3, 2e-3) if dt == torch.float16 else (1e-2, 2e-2)
    np.testing.assert_allclose(host(op), opr, atol=atol, rtol=rtol)
    np.testing.assert_allclose(host(lp)[~empty], lpr[~empty], atol=1e-5, rtol=1e-4)
    O, L = b2a.decode_combine(op, lp, dtype=dt)
    Or, Lr = ora.decode(host(q), host(k), host(v))
    assert_parity(O, L, Or, Lr, NAME[dt])
    O2, L2 = b2a.decode(q, k, v, splits=splits)
    assert torch.equal(O2, O) and torch.equal(L2, L)


def test_combine_matches_oracle_on_random_partials(b2a):
    rng = np.random.default_rng(0)
    op = rng.standard_normal((3, 5, 9, 128)).astype(np.float32)
    lp = (rng.standard_normal((3, 5, 9)) * 4).astype(np.float32)
    lp[0, 0, 3] = -np.inf
    O, L = b2a.decode_combine(torch.from_numpy(op).cuda(), torch.from_numpy(lp).cuda(),
                              dtype=torch.bfloat16)
    Or, Lr = ora.combine(op, lp)
    assert_parity(O, L, Or, Lr, "bfloat16")


def make_paged(B, Hkv, D, page, lens, seed, dt, spare=3):
    """Seeded pool [P, Hkv, page, D] with a random page permutation per sequence."""
    rng = np.random.default_rng(seed)
    npages = -(-np.asarray(lens) // page)
    P = int(npages.sum()) + spare
    perm = rng.permutation(P).astype(np.int32)
    bt = np.zeros((B, int(npages.max())), dtype=np.int32)
    pos = 0
    for b in range(B):
        bt[b, :npages[b]] = perm[pos:pos + npages[b]]
        pos += npages[b]
    kp = ora.seeded_normal((P, Hkv, page, D), seed + 1)
    vp = ora.seeded_normal((P, Hkv, page, D), seed + 2)
    return dev(kp, dt), dev(vp, dt), torch.from_numpy(bt).cuda(), \
        torch.tensor(np.asarray(lens, np.int32)).cuda()


PAGED = [
    # B, H, Hkv, D, page, lens, pages_per_split, dtype
    (4, 32, 8, 128, 16, [1, 15, 16, 17], 4, torch.float16),
    (3, 8, 2, 128, 16, [1000, 64, 513], 8, torch.float16),
    (2, 8, 8, 64, 32, [300, 1], 2, torch.bfloat16),
    (2, 4, 1, 128, 64, [129, 4000], 1, torch.bfloat16),
    (5, 32, 8, 128, 16, [2048, 777, 5, 1024, 3000], 64, torch.float16),
]


@pytest.mark.parametrize("B,H,Hkv,D,page,lens,pps,dt", PAGED, ids=lambda x: str(x))
def test_paged_vs_oracle(b2a, B, H, Hkv, D, page, lens, pps, dt):
    kp, vp, bt, kl = make_paged(B, Hkv, D, page, lens, 11, dt)
    q = dev(ora.seeded_normal((B, H, D), 10), dt)
    O, L = b2a.decode_paged(q, kp, vp, bt, kl, pages_per_split=pps)
    Or, Lr = ora.decode_paged(host(q), host(kp), host(vp), bt.cpu().numpy(), lens)
    assert_parity(O, L, Or, Lr, NAME[dt], 1.0, str(lens))
    torch.cuda.synchronize()
    assert b2a.device_error_flags() == 0


def test_paged_garbage_in_unused_slots_is_ignored(b2a):
    """Slots past a sequence's length may hold anything (here NaN): the result
    must not change."""
    B, H, Hkv, D, page = 2, 8, 2, 128, 16
    lens = [37, 70]
    kp, vp, bt, kl = make_paged(B, Hkv, D, page, lens, 21, torch.float16)
    q = dev(ora.seeded_normal((B, H, D), 20), torch.float16)
    O, L = b2a.decode_paged(q, kp, vp, bt, kl, pages_per_split=4)
    btn = bt.cpu().numpy()
    for b, n in enumerate(lens):
        last = btn[b, (n - 1) // page]
        kp[last, :, n % page or page:] = float("nan")
        vp[last, :, n % page or page:] = float("nan")
    O2, L2 = b2a.decode_paged(q, kp, vp, bt, kl, pages_per_split=4)
    assert torch.equal(O, O2) and torch.equal(L, L2)


def test_config4_full_size_sampled(b2a):
    """Config 4: q [64,32,1,128], K/V [64,8,16384,128] fp16, 16 splits; the oracle
    checks a few batch rows (copied back from the device)."""
    B, H, Hkv, Lkv, D = 64, 32, 8, 16384, 128
    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(B, H, 1, D, device="cuda", generator=g).half()
    k = torch.randn(B, Hkv, Lkv, D, device="cuda", generator=g).half()
    v = torch.randn(B, Hkv, Lkv, D, device="cuda", generator=g).half()
    O, L = b2a.decode(q, k, v, splits=16)
    torch.cuda.synchronize()
    for b in (0, 33, 63):
        Or, Lr = ora.decode(host(q[b:b + 1, :, 0]), host(k[b:b + 1]), host(v[b:b + 1]))
        assert_parity(O[b:b + 1, :, 0], L[b:b + 1, :, 0], Or, Lr, "float16", 1.0, f"b={b}")


def _gather_seq(pool, bt_row, n, page):
    """[1, Hkv, n, D] contiguous copy (on the device) of one sequence's pages."""
    np_ = -(-n // page)
    pages = pool.index_select(0, bt_row[:np_].long())            # [np, Hkv, page, D]
    return pages.permute(1, 0, 2, 3).reshape(1, pool.shape[1], np_ * page, -1)[:, :, :n]


def test_config5a_full_shape_sampled(b2a):
    """Config 5a at its own shape: B=128, H=32, Hkv=8, D=128 fp16, 16-token pages,
    seeded lengths U[512, 32768] (two of them set to a page boundary and one past
    it), pool pages in a seeded random permutation; 64 pages per split (the bench's
    setting).  The oracle checks the longest sequence, the page-boundary ones and
    two more."""
    B, H, Hkv, D, page, pps = 128, 32, 8, 128, 16, 64
    rng = np.random.default_rng(55)
    lens = rng.integers(512, 32768 + 1, size=B).astype(np.int64)
    lens[7], lens[8] = 16384, 16385          # a page boundary and one token past it
    lens[9] = 32768                          # the maximum length: every slot of its last page
    npages = -(-lens // page)
    P = int(npages.sum())
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(77)).to(torch.int32)
    bt = torch.zeros(B, int(npages.max()), dtype=torch.int32)
    pos = 0
    for b in range(B):
        bt[b, :npages[b]] = perm[pos:pos + npages[b]]
        pos += npages[b]
    bt = bt.cuda()
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(5)
    kp = torch.randn(P, Hkv, page, D, device="cuda", generator=g).half()
    vp = torch.randn(P, Hkv, page, D, device="cuda", generator=g).half()
    q = torch.randn(B, H, D, device="cuda", generator=g).half()
    O, L = b2a.decode_paged(q, kp, vp, bt, kl, pages_per_split=pps)
    torch.cuda.synchronize()
    assert b2a.device_error_flags() == 0
    longest = int(np.argmax(lens))
    for b in sorted({longest, 7, 8, 9, 0, 100}):
        n = int(lens[b])
        k = _gather_seq(kp, bt[b], n, page)
        v = _gather_seq(vp, bt[b], n, page)
        Or, Lr = ora.decode(host(q[b:b + 1]), host(k), host(v))
        assert_parity(O[b:b + 1], L[b:b + 1], Or, Lr, "float16", 1.0, f"b={b} len={n}")
    del kp, vp
    torch.cuda.empty_cache()


def test_config5b_full_shape_and_eight_way_shard(b2a):
    """Config 5b at its own shape: B=1, H=32, Hkv=8, KV length 131072 bf16, 32
    splits, through the one-rank path; then the 8-way sequence shard simulated on
    one GPU -- split-KV partials of 8 contiguous 16384-token slices, concatenated
    in sequence order, one combine -- against the same oracle."""
    H, Hkv, L_, D, S = 32, 8, 131072, 128, 32
    g = torch.Generator(device="cuda").manual_seed(55)
    q = torch.randn(1, H, D, device="cuda", generator=g).bfloat16()
    k = torch.randn(1, Hkv, L_, D, device="cuda", generator=g).bfloat16()
    v = torch.randn(1, Hkv, L_, D, device="cuda", generator=g).bfloat16()
    O, L = b2a.decode(q, k, v, splits=S)
    Or, Lr = ora.decode(host(q), host(k), host(v))
    assert_parity(O, L, Or, Lr, "bfloat16", 1.0, "config 5b, one rank")
    world = 8
    sl = L_ // world
    parts = [b2a.decode_splitkv(q, k[:, :, r * sl:(r + 1) * sl].contiguous(),
                                v[:, :, r * sl:(r + 1) * sl].contiguous(), splits=S)
             for r in range(world)]
    op = torch.cat([p[0] for p in parts], dim=2)      # [1, H, world*S, D], sequence order
    lp = torch.cat([p[1] for p in parts], dim=2)
    O8, L8 = b2a.decode_combine(op, lp, dtype=torch.bfloat16)
    assert_parity(O8, L8, Or, Lr, "bfloat16", 1.0, "config 5b, 8 shards")
    torch.cuda.synchronize()
    assert b2a.device_error_flags() == 0
