"""Generate tests/golden/*.npz by running the REFERENCE's own oracle.

Imports `naive_attention` from the reference checkout's ref/naive_attn.py
(Bias92/flashattn-cuda, ref/naive_attn.py:10-38) and evaluates it with torch on
the CPU, in fp32, on seeded inputs -- the inputs are half-cast first, as the
reference's tests do (tests/test_fa3_db_full.py:28-35).  The shape grid is the
reference's own (tests/test_fa3_db_full.py:58-75: full-tile and guarded N,
B=2/H=4, amp=16 stress), plus D=128, bf16-cast inputs, and query-length-1
(decode) cases that the same function evaluates unchanged, and backward
cases from the reference's naive backward (tests/test_backward.py:20-46).

Inputs are stored as raw 16-bit patterns (q, k, v as uint16, with `dtype`
naming float16 or bfloat16); O and L as float32.  The fixtures are committed;
this script needs the reference checkout, so it runs only where that exists:

    python tests/golden/make_golden.py /path/to/reference
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(ref_root: str):
    path = os.path.join(ref_root, "ref", "naive_attn.py")
    spec = importlib.util.spec_from_file_location("ref_naive_attn", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.naive_attention


def load_reference_backward(ref_root: str):
    """The reference's naive backward, tests/test_backward.py:20-46.  That file
    imports a compiled extension at module level, so only the two naive
    functions' source is executed (unchanged), not the module."""
    import ast
    path = os.path.join(ref_root, "tests", "test_backward.py")
    tree = ast.parse(open(path).read())
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef)
            and n.name in ("naive_attention_forward", "naive_attention_backward")]
    ns = {"torch": torch}
    exec(compile(ast.Module(body=keep, type_ignores=[]), path, "exec"), ns)
    return ns["naive_attention_backward"]


def inputs(shape_q, shape_kv, seed, amp, dtype):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal(shape_q, dtype=np.float32) * np.float32(amp))
    k = (rng.standard_normal(shape_kv, dtype=np.float32) * np.float32(amp))
    v = (rng.standard_normal(shape_kv, dtype=np.float32) * np.float32(amp))
    cast = lambda a: torch.from_numpy(a).to(dtype)
    return cast(q), cast(k), cast(v)


PREFILL_CASES = [
    # (name, B, H, N, D, amp, dtype)
    *[(f"n{n}", 1, 1, n, 64, 1.0, torch.float16) for n in (1, 2, 7, 31, 33, 63, 64, 127, 128)],
    ("b2h4n256", 2, 4, 256, 64, 1.0, torch.float16),
    ("n1024", 1, 1, 1024, 64, 1.0, torch.float16),
    ("n255_amp16", 1, 1, 255, 64, 16.0, torch.float16),
    ("d128_n200", 1, 2, 200, 128, 1.0, torch.float16),
    ("bf16_d128_n130", 1, 2, 130, 128, 1.0, torch.bfloat16),
    ("bf16_d64_n96", 2, 1, 96, 64, 1.0, torch.bfloat16),
]

DECODE_CASES = [
    # (name, B, H, L, D, dtype): q [B,H,1,D], K/V [B,H,L,D]
    ("dec_l1000_d128", 1, 2, 1000, 128, torch.float16),
    ("dec_l77_d64", 1, 8, 77, 64, torch.float16),
    ("dec_l513_bf16", 1, 4, 513, 128, torch.bfloat16),
]


BACKWARD_CASES = [
    # (name, B, H, N, D, dtype) -- small cases from the reference's backward grid
    # (tests/test_backward.py:95-105: N 32..2048 at D=64) plus a D=128 bf16 one
    ("bwd_n128", 1, 2, 128, 64, torch.float16),
    ("bwd_n77_d128", 1, 2, 77, 128, torch.bfloat16),
]


def bits(t: torch.Tensor) -> np.ndarray:
    """Raw 16-bit patterns of a half / bfloat16 tensor (lossless, half the size of fp32)."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main(ref_root: str) -> None:
    naive = load_reference(ref_root)
    for i, (name, B, H, N, D, amp, dt) in enumerate(PREFILL_CASES):
        q, k, v = inputs((B, H, N, D), (B, H, N, D), 1000 + i, amp, dt)
        O, L = naive(q.float(), k.float(), v.float())
        np.savez_compressed(os.path.join(HERE, f"prefill_{name}.npz"),
                            q=bits(q), k=bits(k), v=bits(v), O=O.numpy(), L=L.numpy(),
                            dtype=str(dt).split(".")[-1], amp=amp)
    for i, (name, B, H, L_, D, dt) in enumerate(DECODE_CASES):
        q, k, v = inputs((B, H, 1, D), (B, H, L_, D), 2000 + i, 1.0, dt)
        O, L = naive(q.float(), k.float(), v.float())
        np.savez_compressed(os.path.join(HERE, f"decode_{name}.npz"),
                            q=bits(q), k=bits(k), v=bits(v), O=O.numpy(), L=L.numpy(),
                            dtype=str(dt).split(".")[-1])
    naive_bwd = load_reference_backward(ref_root)
    for i, (name, B, H, N, D, dt) in enumerate(BACKWARD_CASES):
        q, k, v = inputs((B, H, N, D), (B, H, N, D), 3000 + i, 1.0, dt)
        rng = np.random.default_rng(4000 + i)
        do = torch.from_numpy(rng.standard_normal((B, H, N, D), dtype=np.float32)).to(dt)
        dQ, dK, dV = naive_bwd(q.float(), k.float(), v.float(), do.float())
        np.savez_compressed(os.path.join(HERE, f"backward_{name}.npz"),
                            q=bits(q), k=bits(k), v=bits(v), do=bits(do), dQ=dQ.numpy(),
                            dK=dK.numpy(), dV=dV.numpy(), dtype=str(dt).split(".")[-1])
    print("wrote", len(PREFILL_CASES) + len(DECODE_CASES) + len(BACKWARD_CASES), "fixtures to", HERE)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("B2A_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py <reference checkout> (or set B2A_REFERENCE_ROOT)")
    main(root)
