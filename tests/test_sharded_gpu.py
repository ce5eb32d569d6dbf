"""KV-sharded decode on GPUs: the CUDA split-KV kernel per rank, then the
exchange -- one kernel over NVLink peer memory (merge, peer stores, combine),
or the collective path (merge, NCCL all-gather, combine); compared with
single-GPU decode and the oracle.  On one GPU the world-size-1 path and
emulated ranks run; the two-rank run needs two GPUs and is skipped otherwise."""
from __future__ import annotations

import os
import socket
import sys
import tempfile
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import assert_parity
from oracle import attention as ora

pytestmark = pytest.mark.gpu

B, H, HKV, L, D = 1, 32, 8, 8192 + 77, 128


def _inputs():
    q = ora.seeded_normal((B, H, D), 1)
    k = ora.seeded_normal((B, HKV, L, D), 2)
    v = ora.seeded_normal((B, HKV, L, D), 3)
    return q, k, v


def test_sharded_world1_equals_decode():
    import b200attn
    from b200attn.sharded import decode_kv_sharded
    q, k, v = (torch.from_numpy(a).to(torch.bfloat16).cuda() for a in _inputs())
    O, Lse = decode_kv_sharded(q, k, v, splits=8)
    O2, L2 = b200attn.decode(q, k, v, splits=8)
    assert torch.equal(O, O2) and torch.equal(Lse, L2)
    Or, Lr = ora.decode(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy())
    assert_parity(O, Lse, Or, Lr, "bfloat16")


@pytest.mark.parametrize("world", [3, 8])
def test_gathered_chunks_combine_in_place(world):
    """The collective path's data path on one GPU: each emulated rank's split-KV
    partials are merged (b2a_decode_merge_splits) into its chunk of one flat
    buffer -- the layout the in-place all-gather leaves on every rank -- and
    combine_kernel reads the chunks where they lie, matching the oracle on the
    whole sequence."""
    import b200attn
    from b200attn.sharded import chunk_views, partials_chunk
    q, k, v = (torch.from_numpy(a).to(torch.bfloat16).cuda() for a in _inputs())
    S = 4
    c = partials_chunk(B, H, D)
    buf = torch.full((world * c,), float("nan"), dtype=torch.float32, device="cuda")
    bnd = np.linspace(0, L, world + 1).astype(int)
    for r in range(world):
        ks = k[:, :, bnd[r]:bnd[r + 1]].contiguous()
        vs = v[:, :, bnd[r]:bnd[r + 1]].contiguous()
        op, lp = b200attn.decode_splitkv(q, ks, vs, splits=S)
        b200attn.decode_merge_splits(op, lp, out=chunk_views(buf[r * c:(r + 1) * c], B, H, D))
    O, Lse = b200attn.decode_combine_ranks(buf, B, H, 1, D, world, c, torch.bfloat16)
    Or, Lr = ora.decode(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy())
    assert_parity(O, Lse, Or, Lr, "bfloat16", 1.0, f"{world} emulated ranks")
    torch.cuda.synchronize()
    assert b200attn.device_error_flags() == 0


def test_merge_splits_is_one_partial():
    """A merged partial is a split partial over the whole range: combining it
    alone gives decode's result."""
    import b200attn
    q, k, v = (torch.from_numpy(a).to(torch.float16).cuda() for a in _inputs())
    op, lp = b200attn.decode_splitkv(q, k, v, splits=7)
    om, lm = b200attn.decode_merge_splits(op, lp)
    O, Lse = b200attn.decode_combine(om.unsqueeze(2), lm.unsqueeze(2), dtype=torch.float16)
    Or, Lr = ora.decode(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy())
    assert_parity(O, Lse, Or, Lr, "float16", 1.0, "merged")
    np.testing.assert_allclose(lm.cpu().numpy(), Lr, rtol=1e-4, atol=1e-5)


def test_exchange_kernel_single_rank_matches_decode():
    """b2a_decode_exchange_combine with world = 1 (its own buffer as the only
    peer), three calls in a row on different queries: each matches the oracle
    within the decode tolerance (merge, delivery into the parity slot, the call
    counters, combine)."""
    import ctypes
    import b200attn
    from b200attn import _lib
    lib = _lib.load()
    q0, k, v = (torch.from_numpy(a).to(torch.bfloat16).cuda() for a in _inputs())
    nbytes = lib.b2a_exchange_bytes(B, H, D, 1)
    own, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
    _lib.check(lib.b2a_exchange_alloc(nbytes, ctypes.byref(own), handle))
    try:
        peers = torch.tensor([own.value], dtype=torch.int64, device="cuda")
        for i in range(3):
            q = q0 * (1.0 + 0.25 * i)
            op, lp = b200attn.decode_splitkv(q, k, v, splits=8)
            O = torch.empty(B, H, D, dtype=torch.bfloat16, device="cuda")
            Lse = torch.empty(B, H, dtype=torch.float32, device="cuda")
            _lib.check(lib.b2a_decode_exchange_combine(
                op.data_ptr(), lp.data_ptr(), peers.data_ptr(), 0, 1, O.data_ptr(),
                Lse.data_ptr(), B, H, 8, D, 1, torch.cuda.current_stream().cuda_stream))
            Or, Lr = ora.decode(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                v.float().cpu().numpy())
            assert_parity(O, Lse, Or, Lr, "bfloat16", 1.0, f"call {i}")
        torch.cuda.synchronize()
        assert b200attn.device_error_flags() == 0
    finally:
        torch.cuda.synchronize()
        lib.b2a_exchange_free(own)


def _worker(rank, world, port, out_dir):
    try:
        root = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..")
        sys.path[:0] = [root, os.path.join(root, "flashattn-cuda_b200")]
        import torch.distributed as dist
        from b200attn.sharded import decode_kv_sharded
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        q, k, v = _inputs()
        bnd = np.linspace(0, L, world + 1).astype(int)
        dev = torch.device("cuda", rank)
        qd = torch.from_numpy(q).to(torch.bfloat16).to(dev)
        ks = torch.from_numpy(np.ascontiguousarray(k[:, :, bnd[rank]:bnd[rank + 1]])).to(torch.bfloat16).to(dev)
        vs = torch.from_numpy(np.ascontiguousarray(v[:, :, bnd[rank]:bnd[rank + 1]])).to(torch.bfloat16).to(dev)
        from b200attn.sharded import close_exchanges
        kb = torch.from_numpy(k).to(torch.bfloat16).float().numpy()
        vb = torch.from_numpy(v).to(torch.bfloat16).float().numpy()
        results = []
        for i in range(3):  # NVLink peer-store exchange, three calls in a row
            qi = qd * (1.0 + 0.25 * i)
            results.append((qi, decode_kv_sharded(qi, ks, vs, splits=8)))
        # the collective path (merge, in-place NCCL all-gather, combine)
        results.append((qd, decode_kv_sharded(qd, ks, vs, splits=8, peer_exchange_path=False)))
        torch.cuda.synchronize()
        import b200attn
        flags = b200attn.device_error_flags()
        close_exchanges()
        dist.destroy_process_group()
        assert flags == 0, flags
        for i, (qi, (O, Lse)) in enumerate(results):
            Or, Lr = ora.decode(qi.float().cpu().numpy(), kb, vb)
            assert_parity(O, Lse, Or, Lr, "bfloat16", 1.0, f"rank {rank} call {i}")
        status = "ok"
    except Exception:
        status = "fail:" + traceback.format_exc()
    with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
        f.write(status)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_two_ranks_nccl():
    s = socket.socket(); s.bind(("127.0.0.1", 0)); port = s.getsockname()[1]; s.close()
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_worker, args=(r, 2, port, d)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
            assert not p.is_alive(), "rank hung"
        for r in range(2):
            assert open(os.path.join(d, f"rank{r}")).read() == "ok"
