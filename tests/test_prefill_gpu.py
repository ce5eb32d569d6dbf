"""Prefill forward on the B200: parity with the oracle and with golden vectors
from the reference's own naive attention, over the reference test grid
(tests/test_fa3_db_full.py:58-75) and the north-star configurations."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
import torch

from conftest import assert_parity, golden_files, load_golden
from oracle import attention as ora

pytestmark = pytest.mark.gpu

TDT = {"float16": torch.float16, "bfloat16": torch.bfloat16}


@pytest.fixture(scope="module")
def b2a():
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    import b200attn
    return b200attn


def dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).cuda()


def host(t):
    return t.float().cpu().numpy()


def seeded(shape_q, shape_kv, seed, amp, dtype):
    """Seeded CPU inputs (identical bits on every device) rounded to `dtype`."""
    q = dev(ora.seeded_normal(shape_q, seed, amp), dtype)
    k = dev(ora.seeded_normal(shape_kv, seed + 1, amp), dtype)
    v = dev(ora.seeded_normal(shape_kv, seed + 2, amp), dtype)
    return q, k, v


@pytest.mark.parametrize("path", golden_files("prefill"), ids=lambda p: os.path.basename(p)[:-4])
def test_golden_prefill(b2a, path):
    g = load_golden(path)
    dt = TDT[g["dtype"]]
    q, k, v = dev(g["q"], dt), dev(g["k"], dt), dev(g["v"], dt)
    O, L = b2a.forward(q, k, v)
    assert O.dtype == dt and L.dtype == torch.float32
    assert_parity(O, L, g["O"], g["L"], g["dtype"], g["amp"], g["name"])
    O2 = b2a.forward_only(q, k, v)
    assert torch.equal(O2, O), "forward_only O must be bitwise equal to forward's O"


REF_GRID = [
    (1, 1, 64), (1, 1, 128), (2, 8, 512), (1, 1, 1024), (1, 1, 2048), (1, 1, 4096),
    (1, 1, 1), (1, 1, 2), (1, 1, 7), (1, 1, 31), (1, 1, 33), (1, 1, 63), (1, 1, 127),
    (1, 1, 4095), (2, 4, 256),
]


@pytest.mark.parametrize("B,H,N", REF_GRID, ids=lambda x: str(x))
def test_reference_grid_fp32_inputs(b2a, B, H, N):
    # fp32 inputs are cast to fp16 like the reference (cuda/flash_attn_fa3_db_full.cu:366)
    q32 = torch.from_numpy(ora.seeded_normal((B, H, N, 64), 42)).cuda()
    k32 = torch.from_numpy(ora.seeded_normal((B, H, N, 64), 43)).cuda()
    v32 = torch.from_numpy(ora.seeded_normal((B, H, N, 64), 44)).cuda()
    O, L = b2a.forward(q32, k32, v32)
    assert O.dtype == torch.float16
    Or, Lr = ora.naive_attention(host(q32.half()), host(k32.half()), host(v32.half()))
    assert_parity(O, L, Or, Lr, "float16", 1.0, f"{B},{H},{N}")
    assert torch.equal(b2a.forward_only(q32, k32, v32), O)


@pytest.mark.parametrize("N,amp", [(2048, 16.0), (4095, 16.0), (1024, 8.0)])
def test_large_logit_stress(b2a, N, amp):
    q, k, v = seeded((1, 1, N, 64), (1, 1, N, 64), 7, amp, torch.float16)
    O, L = b2a.forward(q, k, v)
    Or, Lr = ora.naive_attention(host(q), host(k), host(v))
    assert_parity(O, L, Or, Lr, "float16", amp, f"N={N} amp={amp}")


VARIANTS = [
    # B, H, Hkv, N, D, dtype, causal
    (1, 2, 2, 300, 128, torch.float16, False),
    (1, 2, 2, 300, 128, torch.bfloat16, False),
    (2, 2, 2, 257, 64, torch.bfloat16, True),
    (1, 4, 4, 640, 128, torch.bfloat16, True),
    (1, 3, 3, 129, 64, torch.float16, True),
    (1, 8, 2, 384, 128, torch.float16, False),   # GQA group 4
    (2, 4, 1, 200, 64, torch.bfloat16, True),    # MQA
    (1, 1, 1, 1, 128, torch.bfloat16, True),
]


@pytest.mark.parametrize("B,H,Hkv,N,D,dt,causal", VARIANTS, ids=lambda x: str(x))
def test_variants_vs_oracle(b2a, B, H, Hkv, N, D, dt, causal):
    q, k, v = seeded((B, H, N, D), (B, Hkv, N, D), 100 + N, 1.0, dt)
    O, L = b2a.forward(q, k, v, causal=causal)
    Or, Lr = ora.naive_attention(host(q), host(k), host(v), causal=causal)
    name = "bfloat16" if dt == torch.bfloat16 else "float16"
    assert_parity(O, L, Or, Lr, name, 1.0, f"{B},{H},{Hkv},{N},{D},{causal}")
    assert torch.equal(b2a.forward_only(q, k, v, causal=causal), O)


def test_explicit_scale(b2a):
    q, k, v = seeded((1, 2, 200, 64), (1, 2, 200, 64), 5, 1.0, torch.float16)
    O, L = b2a.forward(q, k, v, scale=0.3)
    Or, Lr = ora.naive_attention(host(q), host(k), host(v), scale=0.3)
    assert_parity(O, L, Or, Lr, "float16")


@pytest.mark.parametrize("cfg", ["config1", "config2"])
def test_headline_configs_full_size(b2a, cfg):
    N = 1024 if cfg == "config1" else 4096
    q, k, v = seeded((1, 8, N, 64), (1, 8, N, 64), 0, 1.0, torch.float16)
    O, L = b2a.forward(q, k, v)
    Or, Lr = ora.naive_attention(host(q), host(k), host(v))
    assert_parity(O, L, Or, Lr, "float16", 1.0, cfg)


def test_config3_causal_bf16_sampled(b2a):
    """Config 3 at full size ([4,32,8192,128] bf16 causal): oracle rows sampled
    from several heads, plus the size-independent row-0 identity O[0] = V[0]."""
    B, H, N, D = 4, 32, 8192, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(B, H, N, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, H, N, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, H, N, D, device="cuda", generator=g).to(torch.bfloat16)
    O, L = b2a.forward(q, k, v, causal=True)
    torch.cuda.synchronize()
    assert torch.isfinite(O).all() and torch.isfinite(L).all()
    # row 0 attends to key 0 only: O = V[0] exactly, L = q0.k0 * scale
    assert torch.equal(O[:, :, 0], v[:, :, 0])
    rows = [0, 1, 127, 128, 129, 4095, 4096, 8190, 8191]
    for b, h in [(0, 0), (1, 17), (3, 31)]:
        qh, kh, vh = host(q[b:b + 1, h:h + 1]), host(k[b:b + 1, h:h + 1]), host(v[b:b + 1, h:h + 1])
        Or, Lr = ora.attention_rows(qh, kh, vh, 0, 0, rows, scale=D ** -0.5, causal=True)
        assert_parity(O[b, h, rows], L[b, h, rows], Or, Lr, "bfloat16", 1.0, f"b{b}h{h}")


def test_misaligned_pointer_rejected(b2a):
    from b200attn import _lib
    lib = _lib.load()
    buf = torch.zeros(2 * 64 * 64 + 8, dtype=torch.float16, device="cuda")
    base = buf.data_ptr() + 2  # 2-byte offset: not 16-byte aligned
    rc = lib.b2a_prefill_fwd(base, base, base, base, None, 1, 1, 1, 64, 64, 0, 0, 0.125,
                             torch.cuda.current_stream().cuda_stream)
    assert rc == 3
    assert b"16-byte aligned" in lib.b2a_last_error()


def test_no_device_errors_recorded(b2a):
    q, k, v = seeded((1, 2, 512, 128), (1, 2, 512, 128), 9, 1.0, torch.bfloat16)
    b2a.forward(q, k, v, causal=True)
    torch.cuda.synchronize()
    assert b2a.device_error_flags() == 0


CROSS = [
    # B, H, Hkv, N, Nk, D, dtype, causal
    (1, 4, 4, 256, 1000, 64, torch.float16, False),
    (1, 4, 2, 129, 700, 128, torch.bfloat16, True),    # a chunk of queries over a longer cache
    (2, 2, 2, 300, 77, 64, torch.float16, False),      # fewer keys than queries
    (1, 8, 8, 64, 4096, 64, torch.float16, True),
    (1, 2, 2, 1, 513, 128, torch.float16, True),       # one query row over a cache
]


@pytest.mark.parametrize("B,H,Hkv,N,Nk,D,dt,causal", CROSS, ids=lambda x: str(x))
def test_cross_attention_nq_ne_nk(b2a, B, H, Hkv, N, Nk, D, dt, causal):
    q, _, _ = seeded((B, H, N, D), (B, Hkv, N, D), 300 + N, 1.0, dt)
    k = dev(ora.seeded_normal((B, Hkv, Nk, D), 400 + Nk), dt)
    v = dev(ora.seeded_normal((B, Hkv, Nk, D), 500 + Nk), dt)
    O, L = b2a.forward(q, k, v, causal=causal)
    Or, Lr = ora.naive_attention(host(q), host(k), host(v), causal=causal)
    name = "bfloat16" if dt == torch.bfloat16 else "float16"
    assert_parity(O, L, Or, Lr, name, 1.0, f"N={N} Nk={Nk}")
    assert torch.equal(b2a.forward_only(q, k, v, causal=causal), O)


def test_causal_needs_nk_at_least_n(b2a):
    q = torch.zeros(1, 1, 128, 64, dtype=torch.float16, device="cuda")
    k = torch.zeros(1, 1, 64, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="Nk >= N"):
        b2a.forward(q, k, k, causal=True)


# Non-causal D = 64 launches whose plain grid would fill less than the GPU run
# split-KV: a cluster of 2-8 CTAs shares each 256-row block, one slice of the
# KV tiles each, merged in-kernel.  The split factor a 148-SM B200 picks is
# noted for each case; the parity bar is the same as for the unsplit kernel.
SPLIT_CASES = [
    # B, H, Hkv, N, Nk, dtype
    (1, 1, 1, 256, 1024, torch.float16),    # 1 block, 8 KV tiles: 8 splits of one tile
    (1, 4, 4, 1000, 1000, torch.bfloat16),  # 16 blocks (the last ragged): 8 splits
    (1, 2, 2, 300, 700, torch.float16),     # 4 blocks, 6 tiles: 2 splits of 3
    (1, 2, 1, 200, 130, torch.bfloat16),    # GQA; split 2 holds one tile of only 2 keys
    (2, 4, 2, 1024, 3000, torch.float16),   # 32 blocks, 24 tiles: 4 splits of 6
]


@pytest.mark.parametrize("B,H,Hkv,N,Nk,dt", SPLIT_CASES, ids=lambda x: str(x))
def test_split_kv_d64(b2a, B, H, Hkv, N, Nk, dt):
    q, _, _ = seeded((B, H, N, 64), (B, Hkv, N, 64), 600 + N, 1.0, dt)
    k = dev(ora.seeded_normal((B, Hkv, Nk, 64), 700 + Nk), dt)
    v = dev(ora.seeded_normal((B, Hkv, Nk, 64), 800 + Nk), dt)
    b2a.device_error_flags()
    O, L = b2a.forward(q, k, v)
    Or, Lr = ora.naive_attention(host(q), host(k), host(v))
    name = "bfloat16" if dt == torch.bfloat16 else "float16"
    assert_parity(O, L, Or, Lr, name, 1.0, f"split-KV N={N} Nk={Nk}")
    assert torch.equal(b2a.forward_only(q, k, v), O)
    torch.cuda.synchronize()
    assert b2a.device_error_flags() == 0


# Causal D = 64 launches split too; ranks whose KV slice lies past a block's
# last visible key have no tile and contribute an empty partial.
SPLIT_CAUSAL_64 = [
    # B, H, Hkv, N, Nk, dtype
    (1, 1, 1, 1024, 1024, torch.float16),   # 4 blocks x 8 ranks; block 0 uses 2 of 8
    (1, 2, 2, 300, 300, torch.bfloat16),    # 4 blocks x 2 ranks, rank 1 of block 0 empty
    (1, 4, 2, 640, 640, torch.float16),     # 12 blocks x 2 ranks; a rank with tile 1 only
    (1, 1, 1, 129, 4096, torch.bfloat16),   # one block x 8 ranks, causal offset 3967
    # GQA with Nk > N under a non-zero causal offset: 2 blocks x 4 heads, the
    # 1100 keys in 9 tiles; in block 0, tile 0 (rows 0-127) sees keys up to
    # 927, tile 1 up to 1055, so some ranks hold tiles for tile 1 only
    (1, 4, 2, 300, 1100, torch.bfloat16),
]


@pytest.mark.parametrize("B,H,Hkv,N,Nk,dt", SPLIT_CAUSAL_64, ids=lambda x: str(x))
def test_split_kv_d64_causal(b2a, B, H, Hkv, N, Nk, dt):
    q, _, _ = seeded((B, H, N, 64), (B, Hkv, N, 64), 1200 + N, 1.0, dt)
    k = dev(ora.seeded_normal((B, Hkv, Nk, 64), 1300 + Nk), dt)
    v = dev(ora.seeded_normal((B, Hkv, Nk, 64), 1400 + Nk), dt)
    b2a.device_error_flags()
    O, L = b2a.forward(q, k, v, causal=True)
    Or, Lr = ora.naive_attention(host(q), host(k), host(v), causal=True)
    name = "bfloat16" if dt == torch.bfloat16 else "float16"
    assert_parity(O, L, Or, Lr, name, 1.0, f"causal split-KV N={N} Nk={Nk}")
    assert torch.equal(b2a.forward_only(q, k, v, causal=True), O)
    torch.cuda.synchronize()
    assert b2a.device_error_flags() == 0


# Dense D = 128 launches are persistent: each CTA walks a static list of
# (head, 256-row block) blocks -- pairs (nqb-1-j, j) per head when there are
# many, a heaviest-first boustrophedon deal of single blocks when there are few,
# one block per item without a mask.  The varlen form of the same kernel runs
# one block per CTA, and with equal lengths its output is bitwise equal to the
# dense one: so every block of every head must be computed exactly once.
SCHEDULE_CASES = [
    # B, H, Hkv, N, causal   (schedule on a 148-SM B200)
    (1, 64, 8, 7936, True),    # pairs: 64 heads x 16 items, the odd block 15 alone
    (2, 4, 2, 3000, True),     # few items: single blocks dealt heaviest first
    (3, 5, 5, 1100, False),    # no mask: one block per item, head-major
]


@pytest.mark.parametrize("B,H,Hkv,N,causal", SCHEDULE_CASES, ids=lambda x: str(x))
def test_persistent_schedule_covers_every_block_once(b2a, B, H, Hkv, N, causal):
    D = 128
    g = torch.Generator(device="cuda").manual_seed(N)
    q = torch.randn(B, H, N, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, N, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, N, D, device="cuda", generator=g).to(torch.bfloat16)
    b2a.device_error_flags()
    O, L = b2a.forward(q, k, v, causal=causal)
    # the same batch through the one-block-per-CTA varlen launch
    pack = lambda t: t.permute(0, 2, 1, 3).reshape(B * N, t.shape[1], D).contiguous()
    cu = torch.arange(0, (B + 1) * N, N, dtype=torch.int32, device="cuda")
    Ov, Lv = b2a.forward_varlen(pack(q), pack(k), pack(v), cu, cu, N, causal=causal)
    assert torch.equal(pack(O), Ov)
    assert torch.equal(L.permute(1, 0, 2).reshape(H, B * N), Lv)
    rows = [0, 255, 256, N // 2, N - 1]
    for b, h in [(0, 0), (B - 1, H - 1)]:
        Or, Lr = ora.attention_rows(host(q), host(k), host(v), b, h, rows, scale=D ** -0.5,
                                    causal=causal)
        assert_parity(O[b, h, rows], L[b, h, rows], Or, Lr, "bfloat16", 1.0, f"b{b}h{h}")
    torch.cuda.synchronize()
    assert b2a.device_error_flags() == 0
