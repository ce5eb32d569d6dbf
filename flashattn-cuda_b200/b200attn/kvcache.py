"""Paged KV cache: a host-side page allocator and the device append.

The pool layout is the one `decode_paged` reads: k_pool, v_pool
[P, Hkv, page_size, D]; sequence b owns the pages listed in row b of an int32
block table, in order.  `PagePool` hands out pages from a free list and keeps
the block table and the per-sequence lengths; `append` writes new tokens
through the CUDA kernel (b2a_kv_append_paged) after making sure every
position they land on has a page.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from . import _lib
from .attention import _DT, _stream


class PagePool:
    """Fixed pool of `num_pages` pages shared by up to `max_seqs` sequences.

    Host bookkeeping only (free list, block table, lengths); the tensors live
    on `device`.  `max_pages` bounds the pages of one sequence (block-table
    width).
    """

    def __init__(self, num_pages: int, page_size: int, num_kv_heads: int, head_dim: int,
                 max_seqs: int, max_pages: int, dtype=torch.float16, device="cuda"):
        if dtype not in _DT:
            raise ValueError("dtype must be torch.float16 or torch.bfloat16")
        self.page_size, self.max_pages = page_size, max_pages
        self.k_pool = torch.zeros(num_pages, num_kv_heads, page_size, head_dim, dtype=dtype,
                                  device=device)
        self.v_pool = torch.zeros_like(self.k_pool)
        self.block_table = torch.full((max_seqs, max_pages), -1, dtype=torch.int32, device=device)
        self.kv_lens = torch.zeros(max_seqs, dtype=torch.int32, device=device)
        self._free: List[int] = list(range(num_pages - 1, -1, -1))
        self._pages: List[List[int]] = [[] for _ in range(max_seqs)]
        self._lens: List[int] = [0] * max_seqs

    @property
    def num_free(self) -> int:
        return len(self._free)

    def reserve(self, seq: int, new_tokens: int) -> None:
        """Make sure sequence `seq` has pages for `new_tokens` more tokens."""
        need = -(-(self._lens[seq] + new_tokens) // self.page_size)
        if need > self.max_pages:
            raise RuntimeError(f"sequence {seq} would need {need} pages > max_pages {self.max_pages}")
        added = []
        while len(self._pages[seq]) < need:
            if not self._free:
                for p in added:  # roll back this reservation
                    self._pages[seq].remove(p)
                    self._free.append(p)
                raise RuntimeError("KV page pool exhausted")
            p = self._free.pop()
            self._pages[seq].append(p)
            added.append(p)
        if added:
            row = torch.tensor(self._pages[seq], dtype=torch.int32)
            self.block_table[seq, :len(row)].copy_(row, non_blocking=False)

    def release(self, seq: int) -> None:
        """Return all pages of `seq` to the pool and reset its length."""
        self._free.extend(reversed(self._pages[seq]))
        self._pages[seq] = []
        self._lens[seq] = 0
        self.block_table[seq].fill_(-1)
        self.kv_lens[seq] = 0

    def lengths(self) -> List[int]:
        return list(self._lens)

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor, seqs: Optional[List[int]] = None):
        """Append k_new, v_new [B, Hkv, T, D] to sequences `seqs` (default 0..B-1)."""
        B, Hkv, T, D = k_new.shape
        seqs = list(range(B)) if seqs is None else list(seqs)
        if len(seqs) != B or v_new.shape != k_new.shape:
            raise RuntimeError("k_new / v_new must be [B, Hkv, T, D] with one sequence per row")
        for s in seqs:
            self.reserve(s, T)
        if seqs == list(range(B)):
            bt, lens = self.block_table[:B], self.kv_lens[:B]
            append_paged(k_new, v_new, self.k_pool, self.v_pool, bt, lens, advance=True)
        else:
            idx = torch.tensor(seqs, dtype=torch.long, device=self.kv_lens.device)
            bt, lens = self.block_table[idx].contiguous(), self.kv_lens[idx].contiguous()
            append_paged(k_new, v_new, self.k_pool, self.v_pool, bt, lens, advance=True)
            self.kv_lens[idx] = lens
        for s in seqs:
            self._lens[s] += T


def append_paged(k_new: torch.Tensor, v_new: torch.Tensor, k_pool: torch.Tensor,
                 v_pool: torch.Tensor, block_table: torch.Tensor, kv_lens: torch.Tensor,
                 advance: bool = True) -> None:
    """Device append of [B, Hkv, T, D] tokens at positions kv_lens[b] + t (see
    b2a_kv_append_paged); with `advance`, kv_lens += T on the device."""
    if not all(t.is_cuda for t in (k_new, v_new, k_pool, v_pool, block_table, kv_lens)):
        raise RuntimeError("KV append tensors must be CUDA tensors")
    B, Hkv, T, D = k_new.shape
    P, Hp, page, Dp = k_pool.shape
    if Hp != Hkv or Dp != D or k_pool.dtype != k_new.dtype:
        raise RuntimeError("k_new must match the pool's KV heads, head dim and dtype")
    lib = _lib.load()
    with torch.cuda.device(k_new.device):
        kn, vn = k_new.contiguous(), v_new.contiguous()
        _lib.check(lib.b2a_kv_append_paged(
            kn.data_ptr(), vn.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
            block_table.data_ptr(), kv_lens.data_ptr(), B, Hkv, T, D, page,
            block_table.shape[1], P, _DT[k_new.dtype], int(bool(advance)),
            _stream(k_new.device)))
