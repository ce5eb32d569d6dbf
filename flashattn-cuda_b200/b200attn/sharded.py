"""Long-context decode with the KV sequence sharded across ranks (one GPU each).

Each rank holds a contiguous slice of the KV cache ([B, Hkv, L/world, D]) and
the full query.  The step is:

  1. local split-KV decode on this rank's slice -> fp32 partials (o, l) for
     S local splits (decode_kernel, no communication);
  2. ONE all-gather of the packed partials [B, H, S, D+1] (o and l side by side)
     over the process group -- NCCL over NVLink/NVSwitch on a B200 box -- into a
     local buffer;
  3. the LSE-weighted combine of all world*S partials on every rank
     (combine_kernel), so every rank ends with the same O and L.

Split boundaries do not change the result: partials over any partition of
the keys combine to the unsharded attention (the online-softmax rescale of
cuda/flash_attn_fa3_db_full.cu:261-284 and :340).  No kernel reads another
GPU's memory; remote partials arrive through the collective.

`local_partials` / `combine` can be replaced (keyword arguments) so that the
exchange and reordering logic can be exercised with CPU tensors and the gloo
backend; the defaults are the CUDA entry points of this package.
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


def gather_partials(o_part: torch.Tensor, l_part: torch.Tensor, group=None,
                    check_shapes: bool = True):
    """All-gather per-rank partials; returns (o_all [B,H,world*S,D], l_all [B,H,world*S])
    with rank r's splits at positions [r*S, (r+1)*S) (sequence order)."""
    world = dist.get_world_size(group)
    B, H, S, D = o_part.shape
    key = (id(group), world, B, H, S, D)
    if check_shapes and key not in _checked_shapes:
        shape = torch.tensor([B, H, S, D], dtype=torch.int64, device=o_part.device)
        shapes = [torch.empty_like(shape) for _ in range(world)]
        dist.all_gather(shapes, shape, group=group)
        for r, s in enumerate(shapes):
            if not torch.equal(s, shape):
                raise ShardMismatchError(
                    f"rank {r} partials have shape {tuple(s.tolist())}, this rank "
                    f"{tuple(shape.tolist())}: every rank must use the same B, H, splits, D")
        _checked_shapes.add(key)
    packed = torch.cat([o_part.float(), l_part.float().unsqueeze(-1)], dim=-1).contiguous()
    out = torch.empty((world * B, H, S, D + 1), dtype=packed.dtype, device=packed.device)
    dist.all_gather_into_tensor(out, packed, group=group)  # rank blocks along dim 0
    out = out.view(world, B, H, S, D + 1).permute(1, 2, 0, 3, 4).reshape(B, H, world * S, D + 1)
    return out[..., :D].contiguous(), out[..., D].contiguous()


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
    """
    from . import attention as A
    had_len = q.dim() == 4
    q3 = q[:, :, 0, :] if had_len else q
    D = q3.shape[-1]
    s = float(D) ** -0.5 if scale is None else float(scale)
    lp = local_partials or (lambda q_, k_, v_, sp_, sc_: A.decode_splitkv(q_, k_, v_, sp_, sc_))
    cb = combine or (lambda o_, l_, dt_: A.decode_combine(o_, l_, dt_))
    o_part, l_part = lp(q3, k_shard, v_shard, splits, s)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        o_all, l_all = gather_partials(o_part, l_part, group, check_shapes)
    else:
        o_all, l_all = o_part, l_part
    dt = out_dtype or (q3.dtype if q3.dtype in (torch.float16, torch.bfloat16) else torch.float16)
    O, L = cb(o_all, l_all, dt)
    if had_len:
        return [O.unsqueeze(2), L.unsqueeze(2)]
    return [O, L]
