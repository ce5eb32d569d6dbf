"""Reference-facing attention API over libb200attn.so.

`forward` and `forward_only` keep the surface of the reference's extension
module (cuda/flash_attn_fa3_db_full.cu:405-418): `forward(Q, K, V)` returns the
list `[O, L]` (O in the compute dtype, L fp32 natural-log logsumexp
[B, H, N]) and `forward_only(Q, K, V)` returns O.  Checks and their messages
follow the reference's host function (cuda/flash_attn_fa3_db_full.cu:352-363);
like it, inputs of any other dtype are cast to fp16 and non-contiguous inputs
are copied (:366-368), and the launch goes on the current stream of Q's device
under a device guard (:365, :380).

Additions over the reference, all opt-in: bf16 inputs compute and return bf16
(the reference would cast them to fp16), D = 128, `causal=True`, an explicit
`scale`, GQA (K/V with fewer heads than Q), a key length Nk different from
the query length N (causal masks aligned to the last key), variable-length
batches packed token-major (`forward_varlen`), and the decode entry points
`decode_splitkv`, `decode_combine`, `decode` and `decode_paged`.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import torch

from . import _lib

_DT = {torch.float16: _lib.B2A_F16, torch.bfloat16: _lib.B2A_BF16}

try:  # CPython binding of b2a_prefill_fwd_kv (same library symbol, cheaper call)
    from . import _fastcall
except ImportError:
    _fastcall = None


def _compute_dtype(t: torch.Tensor) -> torch.dtype:
    return t.dtype if t.dtype in _DT else torch.float16


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    """The current stream of `device` as a raw cudaStream_t (the reference launches on
    at::cuda::getCurrentCUDAStream(), cuda/flash_attn_fa3_db_full.cu:380)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def _as(t: torch.Tensor, dt: torch.dtype) -> torch.Tensor:
    """`t` in dtype `dt`, contiguous (no copy when it already is)."""
    return t if (t.dtype is dt and t.is_contiguous()) else t.to(dt).contiguous()


class _on_device:
    """Device guard that costs nothing when `device` is already current."""

    def __init__(self, device: torch.device):
        self.guard = None if device.index == torch.cuda.current_device() else torch.cuda.device(device)

    def __enter__(self):
        if self.guard is not None:
            self.guard.__enter__()

    def __exit__(self, *exc):
        if self.guard is not None:
            self.guard.__exit__(*exc)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _prefill(Q, K, V, want_L: bool, causal: bool, scale: Optional[float]):
    if not (Q.is_cuda and K.is_cuda and V.is_cuda):
        raise RuntimeError("Q/K/V must be CUDA tensors")
    if Q.dim() != 4:
        raise RuntimeError("Q must be 4D [B, H, N, D]")
    B, H, N, D = Q.shape
    if D not in (64, 128):
        raise RuntimeError("Head dimension must be 64 or 128")
    if N <= 0:
        raise RuntimeError("N must be > 0")
    if (K.dim() != 4 or K.shape != V.shape or K.shape[0] != B or K.shape[3] != D
            or K.shape[1] <= 0 or H % K.shape[1] != 0 or K.shape[2] <= 0):
        raise RuntimeError("K and V must have the same shape as Q (self-attention) up to a KV"
                           " head count that divides H and a key length Nk")
    Nk = K.shape[2]
    if causal and Nk < N:
        raise RuntimeError("causal attention needs Nk >= N (the mask is aligned to the last key)")
    if K.device != Q.device or V.device != Q.device:
        raise RuntimeError("Q/K/V must be on the same device")
    Hkv = K.shape[1]
    dt = _compute_dtype(Q)
    lib = _lib.load()
    with _on_device(Q.device):
        Qc, Kc, Vc = _as(Q, dt), _as(K, dt), _as(V, dt)
        O = torch.empty((B, H, N, D), dtype=dt, device=Q.device)
        L = torch.empty((B, H, N), dtype=torch.float32, device=Q.device) if want_L else None
        s = float(D) ** -0.5 if scale is None else float(scale)
        args = (Qc.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), O.data_ptr(),
                0 if L is None else L.data_ptr(), B, H, Hkv, N, Nk, D, _DT[dt],
                int(bool(causal)), s, _stream(Q.device))
        _lib.check(_fastcall.prefill_fwd_kv(*args) if _fastcall is not None
                   else lib.b2a_prefill_fwd_kv(*args))
    return O, L


def forward(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, causal: bool = False,
            scale: Optional[float] = None) -> list:
    """Attention forward returning [O, L] (reference `forward`)."""
    O, L = _prefill(Q, K, V, True, causal, scale)
    return [O, L]


def forward_only(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, causal: bool = False,
                 scale: Optional[float] = None) -> torch.Tensor:
    """Attention forward returning O only (reference `forward_only`); bitwise equal to forward's O."""
    O, _ = _prefill(Q, K, V, False, causal, scale)
    return O


def forward_varlen(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor,
                   cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor, max_seqlen_q: int,
                   causal: bool = False, scale: Optional[float] = None,
                   want_L: bool = True) -> list:
    """Variable-length attention forward over sequences packed token-major.

    Q [total_q, H, D], K/V [total_k, Hkv, D]; cu_seqlens_q / cu_seqlens_k are
    int32 prefix sums [B+1] starting at 0 (sequence b owns query tokens
    cu_seqlens_q[b] .. cu_seqlens_q[b+1]-1 and the matching keys).
    max_seqlen_q must bound every query length.  Returns [O [total_q, H, D],
    L [H, total_q]] (L is None with want_L=False).  The causal mask is aligned
    per sequence to its last key; a query row that sees no key gets O = 0 and
    L = -inf.  The reference has no varlen form (it requires K and V to have
    Q's shape, cuda/flash_attn_fa3_db_full.cu:358-359).
    """
    for t in (Q, K, V, cu_seqlens_q, cu_seqlens_k):
        if not t.is_cuda:
            raise RuntimeError("Q/K/V must be CUDA tensors")
        if t.device != Q.device:
            raise RuntimeError("Q/K/V must be on the same device")
    if Q.dim() != 3 or K.dim() != 3 or K.shape != V.shape:
        raise RuntimeError("varlen Q must be [total_q, H, D] and K, V [total_k, Hkv, D]")
    total_q, H, D = Q.shape
    total_k, Hkv, Dk = K.shape
    if D not in (64, 128):
        raise RuntimeError("Head dimension must be 64 or 128")
    if Dk != D or Hkv <= 0 or H % Hkv != 0:
        raise RuntimeError("K and V must have Q's head dimension and a KV head count dividing H")
    if (cu_seqlens_q.dim() != 1 or cu_seqlens_q.shape != cu_seqlens_k.shape
            or cu_seqlens_q.numel() < 2):
        raise RuntimeError("cu_seqlens_q and cu_seqlens_k must both be [B+1]")
    if cu_seqlens_q.dtype != torch.int32 or cu_seqlens_k.dtype != torch.int32:
        raise RuntimeError("cu_seqlens must be int32")
    B = cu_seqlens_q.numel() - 1
    dt = _compute_dtype(Q)
    lib = _lib.load()
    with _on_device(Q.device):
        Qc = _as(Q, dt)
        Kc = _as(K, dt)
        Vc = _as(V, dt)
        cq = cu_seqlens_q.contiguous()
        ck = cu_seqlens_k.contiguous()
        O = torch.empty((total_q, H, D), dtype=dt, device=Q.device)
        L = torch.empty((H, total_q), dtype=torch.float32, device=Q.device) if want_L else None
        s = float(D) ** -0.5 if scale is None else float(scale)
        _lib.check(lib.b2a_prefill_fwd_varlen(
            Qc.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), O.data_ptr(), _ptr(L),
            cq.data_ptr(), ck.data_ptr(), B, H, Hkv, total_q, total_k, int(max_seqlen_q), D,
            _DT[dt], int(bool(causal)), s, _stream(Q.device)))
    return [O, L]


def backward(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, O: torch.Tensor,
             dO: torch.Tensor, L: torch.Tensor, causal: bool = False,
             scale: Optional[float] = None) -> list:
    """Gradients [dQ, dK, dV] of the forward (reference `backward(Q, K, V, O, dO, L)`,
    cuda/flash_attn_kernel.cu:417-502).  O and L are `forward`'s outputs; dK, dV
    have K's shape (for GQA they sum over the query heads sharing a KV head)."""
    for t in (Q, K, V, O, dO, L):
        if not t.is_cuda:
            raise RuntimeError("Q/K/V must be CUDA tensors")
    B, H, N, D = Q.shape
    Hkv, Nk = K.shape[1], K.shape[2]
    if D not in (64, 128):
        raise RuntimeError("Head dimension must be 64 or 128")
    if O.shape != Q.shape or dO.shape != Q.shape or L.shape != (B, H, N) or V.shape != K.shape:
        raise RuntimeError("O and dO must have Q's shape, L [B, H, N], V K's shape")
    dt = _compute_dtype(Q)
    lib = _lib.load()
    with _on_device(Q.device):
        Qc, Kc, Vc, Oc, dOc = (_as(t, dt) for t in (Q, K, V, O, dO))
        Lc = L.float().contiguous()
        dQ = torch.empty_like(Qc)
        dK = torch.empty_like(Kc)
        dV = torch.empty_like(Vc)
        ws = torch.empty(int(lib.b2a_backward_workspace_floats(B, H, N, D)), dtype=torch.float32,
                         device=Q.device)
        s = float(D) ** -0.5 if scale is None else float(scale)
        _lib.check(lib.b2a_backward(
            Qc.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), Oc.data_ptr(), dOc.data_ptr(),
            Lc.data_ptr(), dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), ws.data_ptr(),
            B, H, Hkv, N, Nk, D, _DT[dt], int(bool(causal)), s, _stream(Q.device)))
    return [dQ, dK, dV]


# ---------------------------------------------------------------------------- decode

def _decode_q(q: torch.Tensor):
    """Accept q as [B, H, D] or [B, H, 1, D]; return ([B,H,D] view, had_len_dim)."""
    if q.dim() == 4:
        if q.shape[2] != 1:
            raise RuntimeError("decode expects query length 1 ([B, H, 1, D])")
        return q[:, :, 0, :], True
    if q.dim() != 3:
        raise RuntimeError("q must be [B, H, D] or [B, H, 1, D]")
    return q, False


def _check_decode_common(q, k, v):
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("q/K/V must be CUDA tensors")
    if k.device != q.device or v.device != q.device:
        raise RuntimeError("q/K/V must be on the same device")
    if k.shape != v.shape:
        raise RuntimeError("K and V must have the same shape")


def decode_splitkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, splits: int = 16,
                   scale: Optional[float] = None, out=None):
    """Split-KV decode partials.

    q [B, H, D] (or [B, H, 1, D]); k, v [B, Hkv, Lkv, D] contiguous KV cache.
    Returns (o_part fp32 [B, H, splits, D], l_part fp32 [B, H, splits]): per
    split the softmax-normalised output and the natural-log sum of exp.
    `out` = (o_part, l_part): contiguous fp32 tensors of those shapes to write
    into (e.g. views of a collective's buffer) instead of fresh ones.
    """
    q3, _ = _decode_q(q)
    _check_decode_common(q3, k, v)
    if k.dim() != 4:
        raise RuntimeError("K/V must be [B, Hkv, Lkv, D]")
    B, H, D = q3.shape
    Bk, Hkv, Lkv, Dk = k.shape
    if Bk != B or Dk != D or Hkv <= 0 or H % Hkv != 0:
        raise RuntimeError("K/V must be [B, Hkv, Lkv, D] with H a multiple of Hkv")
    dt = _compute_dtype(q3)
    lib = _lib.load()
    with _on_device(q3.device):
        qc = _as(q3, dt)
        kc = _as(k, dt)
        vc = _as(v, dt)
        if out is None:
            o_part = torch.empty((B, H, splits, D), dtype=torch.float32, device=q3.device)
            l_part = torch.empty((B, H, splits), dtype=torch.float32, device=q3.device)
        else:
            o_part, l_part = out
            if (o_part.shape != (B, H, splits, D) or l_part.shape != (B, H, splits)
                    or o_part.dtype != torch.float32 or l_part.dtype != torch.float32
                    or not (o_part.is_contiguous() and l_part.is_contiguous())
                    or o_part.device != q3.device or l_part.device != q3.device):
                raise RuntimeError("out must be contiguous fp32 (o_part [B,H,splits,D], "
                                   "l_part [B,H,splits]) on q's device")
        s = float(D) ** -0.5 if scale is None else float(scale)
        _lib.check(lib.b2a_decode_splitkv(
            qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), o_part.data_ptr(), l_part.data_ptr(),
            B, H, Hkv, Lkv, D, int(splits), _DT[dt], s, _stream(q3.device)))
    return o_part, l_part


def decode_combine(o_part: torch.Tensor, l_part: torch.Tensor,
                   dtype: torch.dtype = torch.float16) -> list:
    """LSE-weighted merge of split partials: returns [O (dtype) [B,H,D], L fp32 [B,H]]."""
    if not (o_part.is_cuda and l_part.is_cuda):
        raise RuntimeError("o_part/l_part must be CUDA tensors")
    if o_part.dim() != 4 or l_part.shape != o_part.shape[:3]:
        raise RuntimeError("o_part must be [B, H, S, D] and l_part [B, H, S]")
    if dtype not in _DT:
        raise RuntimeError("dtype must be torch.float16 or torch.bfloat16")
    B, H, S, D = o_part.shape
    lib = _lib.load()
    with _on_device(o_part.device):
        op = o_part.float().contiguous()
        lp = l_part.float().contiguous()
        O = torch.empty((B, H, D), dtype=dtype, device=o_part.device)
        L = torch.empty((B, H), dtype=torch.float32, device=o_part.device)
        _lib.check(lib.b2a_decode_combine(op.data_ptr(), lp.data_ptr(), O.data_ptr(),
                                          L.data_ptr(), B, H, S, D, _DT[dtype],
                                          _stream(o_part.device)))
    return [O, L]


def decode_merge_splits(o_part: torch.Tensor, l_part: torch.Tensor, out=None):
    """Merge split partials o [B,H,S,D], l [B,H,S] (fp32) into one partial of the
    same form: (o [B,H,D] fp32, normalised, l [B,H] = log sum exp), written into
    `out` = (o, l) when given (b2a_decode_merge_splits)."""
    if not (o_part.is_cuda and l_part.is_cuda):
        raise RuntimeError("o_part/l_part must be CUDA tensors")
    if o_part.dim() != 4 or l_part.shape != o_part.shape[:3]:
        raise RuntimeError("o_part must be [B, H, S, D] and l_part [B, H, S]")
    B, H, S, D = o_part.shape
    lib = _lib.load()
    with _on_device(o_part.device):
        op = o_part.float().contiguous()
        lp = l_part.float().contiguous()
        if out is None:
            om = torch.empty((B, H, D), dtype=torch.float32, device=o_part.device)
            lm = torch.empty((B, H), dtype=torch.float32, device=o_part.device)
        else:
            om, lm = out
            if (om.numel() != B * H * D or lm.numel() != B * H or om.dtype != torch.float32
                    or lm.dtype != torch.float32 or not (om.is_contiguous() and lm.is_contiguous())):
                raise RuntimeError("out must be contiguous fp32 tensors of B*H*D and B*H elements")
        _lib.check(lib.b2a_decode_merge_splits(op.data_ptr(), lp.data_ptr(), om.data_ptr(),
                                               lm.data_ptr(), B, H, S, D,
                                               _stream(o_part.device)))
    return om, lm


def decode_combine_ranks(buf: torch.Tensor, B: int, H: int, splits: int, D: int, ranks: int,
                         rank_stride: int, dtype: torch.dtype = torch.float16) -> list:
    """Combine of the partials of `ranks` ranks gathered into one flat fp32 buffer:
    rank r's chunk starts at buf[r * rank_stride] and holds its o [B,H,splits,D]
    followed by its l [B,H,splits] (b2a_decode_combine_ranks).  Returns
    [O (dtype) [B,H,D], L fp32 [B,H]]."""
    if not buf.is_cuda or buf.dtype != torch.float32 or not buf.is_contiguous():
        raise RuntimeError("buf must be a contiguous fp32 CUDA tensor")
    if buf.numel() < ranks * rank_stride or rank_stride < B * H * splits * (D + 1):
        raise RuntimeError("buf too small for ranks x rank_stride, or rank_stride below "
                           "B*H*splits*(D+1)")
    if dtype not in _DT:
        raise RuntimeError("dtype must be torch.float16 or torch.bfloat16")
    lib = _lib.load()
    with _on_device(buf.device):
        O = torch.empty((B, H, D), dtype=dtype, device=buf.device)
        L = torch.empty((B, H), dtype=torch.float32, device=buf.device)
        base = buf.data_ptr()
        _lib.check(lib.b2a_decode_combine_ranks(base, base + 4 * B * H * splits * D,
                                                O.data_ptr(), L.data_ptr(), B, H, splits,
                                                ranks, rank_stride, D, _DT[dtype],
                                                _stream(buf.device)))
    return [O, L]


def decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, splits: int = 16,
           scale: Optional[float] = None) -> list:
    """Split-KV decode + combine: returns [O, L] shaped like q ([B,H,D] / [B,H,1,D])."""
    q3, had_len = _decode_q(q)
    o_part, l_part = decode_splitkv(q3, k, v, splits, scale)
    O, L = decode_combine(o_part, l_part, _compute_dtype(q3))
    if had_len:
        return [O.unsqueeze(2), L.unsqueeze(2)]
    return [O, L]


def decode_paged(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                 block_table: torch.Tensor, kv_lens: torch.Tensor, pages_per_split: int = 64,
                 scale: Optional[float] = None, scratch: Optional[Sequence[torch.Tensor]] = None
                 ) -> list:
    """Paged-KV decode: returns [O, L] shaped like q.

    k_pool, v_pool: [P, Hkv, page_size, D]; block_table int32 [B, max_pages]
    (page ids of each sequence in order); kv_lens int32 [B] (>= 1 each).
    `scratch` may pass preallocated (o_part, l_part) buffers of shapes
    [B, H, S, D] / [B, H, S] fp32 with S = ceil(max_pages / pages_per_split).
    """
    q3, had_len = _decode_q(q)
    _check_decode_common(q3, k_pool, v_pool)
    if k_pool.dim() != 4:
        raise RuntimeError("k_pool/v_pool must be [P, Hkv, page_size, D]")
    B, H, D = q3.shape
    P, Hkv, page, Dk = k_pool.shape
    if Dk != D or Hkv <= 0 or H % Hkv != 0:
        raise RuntimeError("k_pool must be [P, Hkv, page_size, D] with H a multiple of Hkv")
    if block_table.dim() != 2 or block_table.shape[0] != B or kv_lens.shape != (B,):
        raise RuntimeError("block_table must be [B, max_pages] and kv_lens [B]")
    if not (block_table.is_cuda and kv_lens.is_cuda):
        raise RuntimeError("block_table/kv_lens must be CUDA tensors")
    max_pages = block_table.shape[1]
    S = (max_pages + pages_per_split - 1) // pages_per_split
    dt = _compute_dtype(q3)
    lib = _lib.load()
    with _on_device(q3.device):
        qc = _as(q3, dt)
        kc = _as(k_pool, dt)
        vc = _as(v_pool, dt)
        bt = block_table.to(torch.int32).contiguous()
        kl = kv_lens.to(torch.int32).contiguous()
        if scratch is None:
            o_part = torch.empty((B, H, S, D), dtype=torch.float32, device=q3.device)
            l_part = torch.empty((B, H, S), dtype=torch.float32, device=q3.device)
        else:
            o_part, l_part = scratch
            if o_part.shape != (B, H, S, D) or l_part.shape != (B, H, S):
                raise RuntimeError("scratch buffers have the wrong shape")
        O = torch.empty((B, H, D), dtype=dt, device=q3.device)
        L = torch.empty((B, H), dtype=torch.float32, device=q3.device)
        s = float(D) ** -0.5 if scale is None else float(scale)
        _lib.check(lib.b2a_decode_paged(
            qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), kl.data_ptr(),
            o_part.data_ptr(), l_part.data_ptr(), O.data_ptr(), L.data_ptr(),
            B, H, Hkv, D, page, max_pages, P, int(pages_per_split), _DT[dt], s,
            _stream(q3.device)))
    if had_len:
        return [O.unsqueeze(2), L.unsqueeze(2)]
    return [O, L]


def device_error_flags() -> int:
    """Read and clear the current device's kernel error word (synchronises).

    Bit 0 means a bounded device-side wait timed out; the library reports that
    as B2A_ERR_TIMEOUT, which this function returns as the flag value rather
    than raising (use `check_device()` to raise on it)."""
    import ctypes
    lib = _lib.load()
    v = ctypes.c_uint32(0)
    rc = lib.b2a_device_error(ctypes.byref(v))
    if rc != _lib.B2A_ERR_TIMEOUT:
        _lib.check(rc)
    return int(v.value)


def check_device() -> None:
    """Raise RuntimeError when a kernel since the last check reported an error
    (a timed-out wait, a bad block-table entry, ...); clears the word."""
    flags = device_error_flags()
    if flags:
        raise RuntimeError(f"b200attn: device error word 0x{flags:x} (bit 0: a wait timed out; "
                           "bit 1: bad block-table entry; bit 2: no page for an appended token; "
                           "bit 3: bad cu_seqlens / sequence longer than max_seqlen_q)")


def default_scale(D: int) -> float:
    return 1.0 / math.sqrt(D)
