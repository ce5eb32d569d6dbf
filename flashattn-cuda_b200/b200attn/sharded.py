"""Long-context decode with the KV sequence sharded across ranks (one GPU each).

Each rank holds a contiguous slice of the KV cache ([B, Hkv, L/world, D]) and
the full query.  A step is three launches per rank:

  1. local split-KV decode on this rank's slice (decode_kernel), writing its
     fp32 partials -- o [B, H, S, D] then l [B, H, S] -- straight into this
     rank's chunk of a flat gather buffer [world * chunk];
  2. ONE in-place all-gather of the chunks over the process group -- NCCL over
     NVLink/NVSwitch on a B200 box -- so every rank holds every chunk in its
     own memory;
  3. the LSE-weighted combine of all world*S partials (combine_kernel reading
     the gathered chunks where they lie, b2a_decode_combine_ranks), so every
     rank ends with the same O and L.

There is no packing, reordering or slicing copy between the steps.  Split
boundaries do not change the result: partials over any partition of the keys
combine to the unsharded attention (the online-softmax rescale of
cuda/flash_attn_fa3_db_full.cu:261-284 and :340).  No kernel reads another
GPU's memory; remote partials arrive through the collective.

`local_partials` / `combine` can be replaced (keyword arguments) so that the
exchange logic can be exercised with CPU tensors and the gloo backend; the
defaults are the CUDA entry points of this package.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


class ShardMismatchError(RuntimeError):
    """Ranks disagree on the partial shapes (batch, heads, splits or head dim)."""


# (group, shape) pairs whose agreement across ranks has been checked.  The check
# costs a collective and a host synchronisation, so it runs once per shape, not
# once per decode step.
_checked_shapes: set = set()


def partials_chunk(B: int, H: int, S: int, D: int) -> int:
    """Floats of one rank's chunk of the gather buffer: o [B,H,S,D] then l
    [B,H,S], rounded up to 64 floats so that every chunk starts 256-byte
    aligned."""
    n = B * H * S * (D + 1)
    return (n + 63) // 64 * 64


def chunk_views(chunk: torch.Tensor, B: int, H: int, S: int, D: int):
    """(o [B,H,S,D], l [B,H,S]) views of one rank's chunk."""
    n = B * H * S * D
    return chunk[:n].view(B, H, S, D), chunk[n:n + B * H * S].view(B, H, S)


def unpack_gathered(buf: torch.Tensor, world: int, B: int, H: int, S: int, D: int):
    """(o_all [B,H,world*S,D], l_all [B,H,world*S]) in sequence order, copied out
    of a gathered buffer (for combine functions that want the plain layout)."""
    c = partials_chunk(B, H, S, D)
    parts = [chunk_views(buf[r * c:(r + 1) * c], B, H, S, D) for r in range(world)]
    return torch.cat([p[0] for p in parts], dim=2), torch.cat([p[1] for p in parts], dim=2)


def _check_shapes(B, H, S, D, device, group):
    world = dist.get_world_size(group)
    key = (id(group), world, B, H, S, D)
    if key in _checked_shapes:
        return
    shape = torch.tensor([B, H, S, D], dtype=torch.int64, device=device)
    shapes = [torch.empty_like(shape) for _ in range(world)]
    dist.all_gather(shapes, shape, group=group)
    for r, s in enumerate(shapes):
        if not torch.equal(s, shape):
            raise ShardMismatchError(
                f"rank {r} partials have shape {tuple(s.tolist())}, this rank "
                f"{tuple(shape.tolist())}: every rank must use the same B, H, splits, D")
    _checked_shapes.add(key)


def decode_kv_sharded(q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
                      group=None, splits: int = 16, scale: Optional[float] = None,
                      out_dtype: Optional[torch.dtype] = None, check_shapes: bool = True,
                      local_partials: Optional[Callable] = None,
                      combine: Optional[Callable] = None) -> list:
    """Decode with the KV sequence sharded across the ranks of `group`.

    q [B, H, D] (or [B, H, 1, D]) identical on every rank; k_shard, v_shard
    [B, Hkv, L_r, D] this rank's contiguous slice, in rank order along the
    sequence.  Every rank must use the same `splits`.  Returns [O, L] like
    `decode` on the whole sequence, on every rank.

    Hooks: local_partials(q, k, v, splits, scale, out) writes this rank's
    partials into out = (o [B,H,S,D], l [B,H,S]); combine(buf, world, B, H, S,
    D, dtype) returns [O, L] from the gathered buffer (chunks of
    partials_chunk(B, H, S, D) floats, see chunk_views).
    """
    from . import attention as A
    had_len = q.dim() == 4
    q3 = q[:, :, 0, :] if had_len else q
    B, H, D = q3.shape
    S = int(splits)
    s = float(D) ** -0.5 if scale is None else float(scale)
    dt = out_dtype or (q3.dtype if q3.dtype in (torch.float16, torch.bfloat16) else torch.float16)
    lp = local_partials or (
        lambda q_, k_, v_, sp_, sc_, out_: A.decode_splitkv(q_, k_, v_, sp_, sc_, out=out_))
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        # one rank: no exchange; identical to decode()
        o_part = torch.empty((B, H, S, D), dtype=torch.float32, device=q3.device)
        l_part = torch.empty((B, H, S), dtype=torch.float32, device=q3.device)
        lp(q3, k_shard, v_shard, S, s, (o_part, l_part))
        if combine is not None:
            buf = torch.cat([o_part.reshape(-1), l_part.reshape(-1)])
            O, L = combine(buf, 1, B, H, S, D, dt)
        else:
            O, L = A.decode_combine(o_part, l_part, dt)
    else:
        if check_shapes:
            _check_shapes(B, H, S, D, q3.device, group)
        rank = dist.get_rank(group)
        c = partials_chunk(B, H, S, D)
        buf = torch.empty(world * c, dtype=torch.float32, device=q3.device)
        mine = buf[rank * c:(rank + 1) * c]
        lp(q3, k_shard, v_shard, S, s, chunk_views(mine, B, H, S, D))
        dist.all_gather_into_tensor(buf, mine, group=group)   # in place: rank chunks in order
        if combine is not None:
            O, L = combine(buf, world, B, H, S, D, dt)
        else:
            O, L = A.decode_combine_ranks(buf, B, H, S, D, world, c, dt)
    if had_len:
        return [O.unsqueeze(2), L.unsqueeze(2)]
    return [O, L]
