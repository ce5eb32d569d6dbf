"""Parity with the reference's own kernel: fa3db_full_fwd_kernel
(cuda/flash_attn_fa3_db_full.cu, compiled unmodified for sm_100a into
oracle/_ref/ by oracle/build_ref.py) and b200attn run on identical inputs over
the reference's test grid (tests/test_fa3_db_full.py:58-75).  Both are held to
the reference test's tolerance against the fp64 oracle, and to twice that
against each other."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_parity, parity_tol
from oracle import attention as ora
from oracle.build_ref import load_built

pytestmark = pytest.mark.gpu

GRID = [(1, 1, 64), (1, 1, 128), (2, 8, 512), (1, 1, 1024), (1, 1, 4096), (1, 1, 1),
        (1, 1, 7), (1, 1, 33), (1, 1, 127), (1, 1, 4095), (2, 4, 256), (1, 8, 2048)]


@pytest.fixture(scope="module")
def ref_mod():
    mod = load_built()
    if mod is None:
        pytest.skip("oracle/_ref/flash_attn_fa3_db_full.so not built (python oracle/build_ref.py)")
    return mod


@pytest.mark.parametrize("B,H,N", GRID, ids=lambda x: str(x))
def test_matches_reference_kernel(ref_mod, B, H, N):
    import b200attn
    q, k, v = (torch.from_numpy(ora.seeded_normal((B, H, N, 64), s)).half().cuda()
               for s in (42, 43, 44))
    O, L = b200attn.forward(q, k, v)
    Oref, Lref = ref_mod.forward(q, k, v)
    torch.cuda.synchronize()
    Oo, Lo = ora.naive_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                 v.float().cpu().numpy())
    assert_parity(O, L, Oo, Lo, "float16", 1.0, "b200attn vs oracle")
    assert_parity(Oref, Lref, Oo, Lo, "float16", 1.0, "reference kernel vs oracle")
    atol, rtol = parity_tol("float16")
    np.testing.assert_allclose(O.float().cpu().numpy(), Oref.float().cpu().numpy(),
                               atol=2 * atol, rtol=2 * rtol)
    np.testing.assert_allclose(L.cpu().numpy(), Lref.cpu().numpy(), atol=2e-5, rtol=2e-4)
    assert torch.equal(ref_mod.forward_only(q, k, v), Oref)


@pytest.mark.parametrize("N", [1024, 2048, 4096])
def test_paired_timing_against_reference_kernel(ref_mod, N):
    """The rebuilt reference kernel as a measured bar, with the reference's own
    protocol (bench/bench_fa3_headline.py:24-85): B=1 H=8 D=64 fp16 forward()+L,
    CUDA events, 10 reps whose order alternates between the two kernels, median
    of the per-rep times.  Prints one JSON line; b200attn must be faster."""
    import json
    import statistics
    import b200attn
    q, k, v = (torch.from_numpy(ora.seeded_normal((1, 8, N, 64), s)).half().cuda()
               for s in (42, 43, 44))
    runs = {"b200attn": lambda: b200attn.forward(q, k, v),
            "reference": lambda: ref_mod.forward(q, k, v)}
    for f in runs.values():
        for _ in range(5):
            f()
    torch.cuda.synchronize()
    times = {name: [] for name in runs}
    iters = 20
    for rep in range(10):
        order = list(runs) if rep % 2 == 0 else list(runs)[::-1]
        for name in order:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for _ in range(iters):
                runs[name]()
            e1.record()
            torch.cuda.synchronize()
            times[name].append(e0.elapsed_time(e1) / iters)
    med = {n: statistics.median(t) for n, t in times.items()}
    flops = 4 * 8 * N * N * 64
    print(json.dumps({"shape": f"B=1 H=8 N={N} D=64 fp16",
                      **{f"{n}_ms": round(m, 5) for n, m in med.items()},
                      **{f"{n}_tflops": round(flops / m / 1e9, 1) for n, m in med.items()},
                      "speedup": round(med["reference"] / med["b200attn"], 2)}))
    assert med["b200attn"] < med["reference"]
