"""Long-context decode with the KV sequence sharded across ranks (one GPU each).

Each rank holds a contiguous slice of the KV cache ([B, Hkv, L/world, D]) and
the full query.  A step per rank is:

  1. local split-KV decode on this rank's slice (decode_kernel) -> fp32
     partials (o, l) for S local splits;
  2. merge of those S partials into ONE partial of the same form, the rank's
     contribution: o [B, H, D] then l [B, H] -- B*H*(D+1) floats, 16.5 KB at
     B=1, H=32, D=128, instead of S times that;
  3. exchange of the merged partials so that every rank holds all of them;
  4. the LSE-weighted combine of the world partials, so every rank ends with
     the same O and L.

On CUDA tensors steps 2-4 are ONE kernel over NVLink peer memory
(PeerExchange, b2a_decode_exchange_combine): the merged partial is stored
straight into every rank's exchange buffer, and each rank combines once all
have arrived -- two launches per step, no collective-library call.  The
collective path (peer_exchange_path=False, or any hook) runs step 2 as
combine_kernel's fp32 mode writing into this rank's chunk of a flat buffer,
step 3 as one in-place all_gather_into_tensor (NCCL on a B200 box, gloo on
CPU) and step 4 as combine_kernel reading the gathered chunks where they lie.

There is no packing, reordering or slicing copy between the steps.  Split
boundaries do not change the result: partials over any partition of the keys
combine to the unsharded attention (the online-softmax rescale of
cuda/flash_attn_fa3_db_full.cu:261-284 and :340), and a merged partial is one
such partial.  No kernel reads another GPU's memory: partials arrive by the
collective, or by the sending rank's own stores into the receiver's buffer.

`local_partials` / `merge` / `combine` can be replaced (keyword arguments) so
that the exchange logic can be exercised with CPU tensors and the gloo
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


def partials_chunk(B: int, H: int, D: int) -> int:
    """Floats of one rank's chunk of the gather buffer: its merged o [B,H,D] then
    l [B,H], rounded up to 64 floats so that every chunk starts 256-byte
    aligned."""
    n = B * H * (D + 1)
    return (n + 63) // 64 * 64


def chunk_views(chunk: torch.Tensor, B: int, H: int, D: int):
    """(o [B,H,D], l [B,H]) views of one rank's chunk."""
    n = B * H * D
    return chunk[:n].view(B, H, D), chunk[n:n + B * H].view(B, H)


def unpack_gathered(buf: torch.Tensor, world: int, B: int, H: int, D: int):
    """(o_all [B,H,world,D], l_all [B,H,world]) in sequence order, copied out of a
    gathered buffer (for combine functions that want the split layout)."""
    c = partials_chunk(B, H, D)
    parts = [chunk_views(buf[r * c:(r + 1) * c], B, H, D) for r in range(world)]
    return torch.stack([p[0] for p in parts], dim=2), torch.stack([p[1] for p in parts], dim=2)


class PeerExchange:
    """The exchange buffers of KV-sharded decode over NVLink peer memory.

    Every rank of `group` allocates one buffer (b2a_exchange_alloc), the ranks
    swap their CUDA IPC handles through the process group, and each maps the
    others' buffers (b2a_exchange_open).  `combine(o_part, l_part, dtype)` is
    then one kernel per step (b2a_decode_exchange_combine): merge of the rank's
    split partials, peer stores of the merged partial into every rank's buffer,
    a bounded wait for the others', and the combine.  Collective to construct
    and to close; calls on one rank must be ordered (one stream) and made by
    every rank in the same sequence with the same B, H, D.
    """

    def __init__(self, group, B: int, H: int, D: int, device: torch.device):
        import ctypes
        from . import _lib
        self.lib = lib = _lib.load()
        self.group = group
        self.B, self.H, self.D = B, H, D
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        self._opened: list = []
        self._own = None
        with torch.cuda.device(device):
            nbytes = lib.b2a_exchange_bytes(B, H, D, self.world)
            own = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(64)
            _lib.check(lib.b2a_exchange_alloc(nbytes, ctypes.byref(own), handle))
            self._own = own.value
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            ptrs = []
            try:
                for r, h in enumerate(handles):
                    if r == self.rank:
                        ptrs.append(self._own)
                        continue
                    p = ctypes.c_void_p()
                    _lib.check(lib.b2a_exchange_open(ctypes.create_string_buffer(h, 64),
                                                     ctypes.byref(p)))
                    self._opened.append(p.value)
                    ptrs.append(p.value)
            except Exception:
                self.close(barrier=False)
                raise
            self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)
        dist.barrier(group=group)

    def combine(self, o_part: torch.Tensor, l_part: torch.Tensor, dtype: torch.dtype) -> list:
        from . import _lib
        from .attention import _DT, _stream
        B, H, S, D = o_part.shape
        if (B, H, D) != (self.B, self.H, self.D):
            raise ShardMismatchError("partials do not match the exchange's B, H, D")
        O = torch.empty((B, H, D), dtype=dtype, device=o_part.device)
        L = torch.empty((B, H), dtype=torch.float32, device=o_part.device)
        _lib.check(self.lib.b2a_decode_exchange_combine(
            o_part.data_ptr(), l_part.data_ptr(), self.peers.data_ptr(), self.rank, self.world,
            O.data_ptr(), L.data_ptr(), B, H, S, D, _DT[dtype], _stream(o_part.device)))
        return [O, L]

    def close(self, barrier: bool = True) -> None:
        """Unmap the peers' buffers and free this rank's (after every rank is done)."""
        if barrier:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                self.lib.b2a_exchange_close(p)
            self._opened = []
            if barrier:
                dist.barrier(group=self.group)
            if self._own is not None:
                self.lib.b2a_exchange_free(self._own)
                self._own = None


# (group, world, B, H, D, device) -> PeerExchange, made on first use
_exchanges: dict = {}


def peer_exchange(group, B: int, H: int, D: int, device: torch.device) -> PeerExchange:
    """The PeerExchange for this group and shape, made (collectively) on first use."""
    key = (id(group), dist.get_world_size(group), B, H, D, str(device))
    if key not in _exchanges:
        _exchanges[key] = PeerExchange(group, B, H, D, device)
    return _exchanges[key]


def close_exchanges() -> None:
    """Close every PeerExchange made by peer_exchange (collective)."""
    for ex in list(_exchanges.values()):
        ex.close()
    _exchanges.clear()


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
                      merge: Optional[Callable] = None,
                      combine: Optional[Callable] = None,
                      peer_exchange_path: bool = True) -> list:
    """Decode with the KV sequence sharded across the ranks of `group`.

    q [B, H, D] (or [B, H, 1, D]) identical on every rank; k_shard, v_shard
    [B, Hkv, L_r, D] this rank's contiguous slice, in rank order along the
    sequence.  Every rank must use the same `splits`.  Returns [O, L] like
    `decode` on the whole sequence, on every rank.

    On CUDA tensors with more than one rank the exchange is one kernel over
    NVLink peer memory (PeerExchange); peer_exchange_path=False, or any hook,
    uses the collective path instead.

    Hooks: local_partials(q, k, v, splits, scale) -> (o [B,H,S,D], l [B,H,S]);
    merge(o, l, out) writes the merged partial into out = (o [B,H,D], l [B,H]);
    combine(buf, world, B, H, D, dtype) -> [O, L] from the gathered buffer
    (chunks of partials_chunk(B, H, D) floats, see chunk_views).
    """
    from . import attention as A
    had_len = q.dim() == 4
    q3 = q[:, :, 0, :] if had_len else q
    B, H, D = q3.shape
    S = int(splits)
    s = float(D) ** -0.5 if scale is None else float(scale)
    dt = out_dtype or (q3.dtype if q3.dtype in (torch.float16, torch.bfloat16) else torch.float16)
    lp = local_partials or (lambda q_, k_, v_, sp_, sc_: A.decode_splitkv(q_, k_, v_, sp_, sc_))
    mg = merge or (lambda o_, l_, out_: A.decode_merge_splits(o_, l_, out=out_))
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    o_part, l_part = lp(q3, k_shard, v_shard, S, s)
    if world == 1:
        # one rank: no exchange; identical to decode()
        if combine is not None:
            buf = torch.empty(partials_chunk(B, H, D), dtype=torch.float32, device=q3.device)
            mg(o_part, l_part, chunk_views(buf, B, H, D))
            O, L = combine(buf, 1, B, H, D, dt)
        else:
            O, L = A.decode_combine(o_part, l_part, dt)
    elif (peer_exchange_path and q3.is_cuda and local_partials is None and merge is None
          and combine is None):
        if check_shapes:
            _check_shapes(B, H, S, D, q3.device, group)
        O, L = peer_exchange(group, B, H, D, q3.device).combine(o_part, l_part, dt)
    else:
        if check_shapes:
            _check_shapes(B, H, S, D, q3.device, group)
        rank = dist.get_rank(group)
        c = partials_chunk(B, H, D)
        buf = torch.empty(world * c, dtype=torch.float32, device=q3.device)
        mine = buf[rank * c:(rank + 1) * c]
        mg(o_part, l_part, chunk_views(mine, B, H, D))
        dist.all_gather_into_tensor(buf, mine, group=group)   # in place: rank chunks in order
        if combine is not None:
            O, L = combine(buf, world, B, H, D, dt)
        else:
            O, L = A.decode_combine_ranks(buf, B, H, 1, D, world, c, dt)
    if had_len:
        return [O.unsqueeze(2), L.unsqueeze(2)]
    return [O, L]
