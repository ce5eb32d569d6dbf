"""CUDA-graph-captured decode steps.

A decode step is a few short launches: the split-KV kernel, on multi-GPU runs
an NCCL all-gather of the partials, and the combine kernel.  At small batch
their launch and collective latency rivals the HBM time.  `CapturedDecode`
records one step into a CUDA graph over static buffers; each later step only
copies the new query into the static input and replays the graph, a single
launch.

The KV cache tensors are captured by address: keep them alive and update
them in place (appending tokens changes `Lkv`, which needs a new capture).
"""
from __future__ import annotations

from typing import Optional

import torch


class CapturedDecode:
    """One decode step (split-KV + [all-gather] + combine) as a CUDA graph.

    q: [B, H, D] or [B, H, 1, D]; k, v: [B, Hkv, Lkv, D] on this rank (the
    rank's contiguous KV slice when `sharded`).  With `sharded=True` the step
    is b200attn.sharded.decode_kv_sharded over `group`, otherwise decode.
    """

    def __init__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, splits: int = 16,
                 scale: Optional[float] = None, sharded: bool = False, group=None,
                 warmup: int = 3):
        from . import attention as A
        from .sharded import decode_kv_sharded
        self.q = q.clone()
        self.k, self.v = k, v
        if sharded:
            def step():
                return decode_kv_sharded(self.q, self.k, self.v, group=group, splits=splits,
                                         scale=scale)
        else:
            def step():
                return A.decode(self.q, self.k, self.v, splits=splits, scale=scale)
        side = torch.cuda.Stream(device=q.device)
        side.wait_stream(torch.cuda.current_stream(q.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):  # library set-up, NCCL communicator, shape checks
                step()
        torch.cuda.current_stream(q.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = step()

    def __call__(self, q: Optional[torch.Tensor] = None) -> list:
        """Run one step (optionally on a new query); returns the static [O, L]."""
        if q is not None:
            self.q.copy_(q, non_blocking=True)
        self.graph.replay()
        return self.out
