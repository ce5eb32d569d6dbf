"""KV-sharded decode (config 5b's exchange step) on CPU ranks with the gloo
backend, on the collective form of the exchange.  The per-rank partials, the
merge and the combine come from the oracle here (the CUDA kernels need a GPU),
so these tests cover the host-side logic: the sequence split, the per-rank
merge into its chunk, the in-place all-gather of the chunks, their order,
shape agreement across ranks, and what a surviving rank sees when a
peer dies before the collective (a bounded error, never a hang)."""
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
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import attention as ora

B, H, HKV, L, D = 2, 8, 2, 301, 64


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_partials(q, k, v, splits, scale):
    op, lp = ora.decode_splitkv_partials(q.numpy(), k.numpy(), v.numpy(), splits, scale)
    return torch.from_numpy(op).float(), torch.from_numpy(lp).float()


def _oracle_merge(o, l, out):
    # a merged partial is the combine's O (normalised) and L = log sum exp
    O, Lse = ora.combine(o.numpy(), l.numpy())
    out[0].copy_(torch.from_numpy(O))
    out[1].copy_(torch.from_numpy(Lse))


def _oracle_combine(buf, world, B_, H_, D_, dt):
    from b200attn.sharded import unpack_gathered
    o, l = unpack_gathered(buf, world, B_, H_, D_)
    O, Lse = ora.combine(o.numpy(), l.numpy())
    return torch.from_numpy(O).float(), torch.from_numpy(Lse).float()


def _worker(rank, world, port, mode, out_dir):
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..",
                                    "flashattn-cuda_b200"))
    from b200attn.sharded import ShardMismatchError, decode_kv_sharded
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    status = "ok"
    try:
        q = ora.seeded_normal((B, H, D), 1)
        k = ora.seeded_normal((B, HKV, L, D), 2)
        v = ora.seeded_normal((B, HKV, L, D), 3)
        bounds = np.linspace(0, L, world + 1).astype(int)      # uneven shards are fine
        ks = torch.from_numpy(np.ascontiguousarray(k[:, :, bounds[rank]:bounds[rank + 1]]))
        vs = torch.from_numpy(np.ascontiguousarray(v[:, :, bounds[rank]:bounds[rank + 1]]))
        splits = 3
        if mode == "mismatch" and rank == 1:
            splits = 4
        if mode == "dead" and rank == 1:
            os._exit(0)                                        # leaves before the collective
        O, Lse = decode_kv_sharded(torch.from_numpy(q), ks, vs, splits=splits,
                                   local_partials=_oracle_partials, merge=_oracle_merge,
                                   combine=_oracle_combine)
        Or, Lr = ora.decode(q, k, v)
        np.testing.assert_allclose(O.numpy(), Or, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(Lse.numpy(), Lr, rtol=1e-6, atol=1e-6)
    except ShardMismatchError:
        status = "mismatch"
    except RuntimeError as e:   # the collective failed because a peer is gone
        status = "peer_error" if mode == "dead" else "fail:" + traceback.format_exc()
    except Exception:
        status = "fail:" + traceback.format_exc()
    with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
        f.write(status)
    if mode != "dead":
        dist.destroy_process_group()
    os._exit(0)


def _run(world, mode):
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_worker, args=(r, world, port, mode, d))
                 for port in [_free_port()] for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=90)
            if p.is_alive():
                p.kill()
                raise AssertionError("a rank did not finish (hang)")
        out = {}
        for r in range(world):
            path = os.path.join(d, f"rank{r}")
            out[r] = open(path).read() if os.path.exists(path) else None
        return out


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_decode_matches_unsharded(world):
    out = _run(world, "ok")
    assert all(v == "ok" for v in out.values()), out


def test_ranks_with_different_splits_are_rejected():
    out = _run(2, "mismatch")
    assert out == {0: "mismatch", 1: "mismatch"}, out


def test_dead_peer_gives_bounded_error():
    out = _run(2, "dead")
    assert out[1] is None          # rank 1 left before the collective
    assert out[0] == "peer_error", out
