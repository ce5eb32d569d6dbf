"""KV-sharded decode on GPUs: the CUDA split-KV kernel per rank, NCCL
all-gather of the partials, CUDA combine; compared with single-GPU decode and
the oracle.  On one GPU the world-size-1 path (no collective) runs; the
two-rank NCCL run needs two GPUs and is skipped otherwise."""
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
    """The KV-sharded step's data path on one GPU: each emulated rank's split-KV
    kernel writes its partials into its chunk of one flat buffer (the layout the
    in-place all-gather leaves on every rank), and combine_kernel reads the
    chunks where they lie -- no packing or reordering copy -- matching the
    oracle on the whole sequence."""
    import b200attn
    from b200attn.attention import decode_combine_ranks
    from b200attn.sharded import chunk_views, partials_chunk
    q, k, v = (torch.from_numpy(a).to(torch.bfloat16).cuda() for a in _inputs())
    S = 4
    c = partials_chunk(B, H, S, D)
    buf = torch.full((world * c,), float("nan"), dtype=torch.float32, device="cuda")
    bnd = np.linspace(0, L, world + 1).astype(int)
    for r in range(world):
        ks = k[:, :, bnd[r]:bnd[r + 1]].contiguous()
        vs = v[:, :, bnd[r]:bnd[r + 1]].contiguous()
        b200attn.decode_splitkv(q, ks, vs, splits=S, out=chunk_views(buf[r * c:(r + 1) * c],
                                                                     B, H, S, D))
    O, Lse = decode_combine_ranks(buf, B, H, S, D, world, c, torch.bfloat16)
    Or, Lr = ora.decode(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy())
    assert_parity(O, Lse, Or, Lr, "bfloat16", 1.0, f"{world} emulated ranks")
    torch.cuda.synchronize()
    assert b200attn.device_error_flags() == 0


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
        O, Lse = decode_kv_sharded(qd, ks, vs, splits=8)
        torch.cuda.synchronize()
        dist.destroy_process_group()
        kb = torch.from_numpy(k).to(torch.bfloat16).float().numpy()
        vb = torch.from_numpy(v).to(torch.bfloat16).float().numpy()
        Or, Lr = ora.decode(qd.float().cpu().numpy(), kb, vb)
        assert_parity(O, Lse, Or, Lr, "bfloat16", 1.0, f"rank {rank}")
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
