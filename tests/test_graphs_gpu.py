"""CUDA-graph-captured decode steps: each replay, on new query contents, matches
the CPU oracle within the decode tolerance, and is bitwise equal to the eager
call of the same entry point."""
from __future__ import annotations

import pytest
import torch

from conftest import assert_parity
from oracle import attention as ora

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("sharded", [False, True])
def test_captured_decode_matches_oracle(sharded):
    import b200attn
    from b200attn.graphs import CapturedDecode
    from b200attn.sharded import decode_kv_sharded
    g = torch.Generator(device="cuda").manual_seed(7)
    q0 = torch.randn(2, 32, 1, 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(2, 8, 3000, 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(2, 8, 3000, 128, device="cuda", generator=g).to(torch.bfloat16)
    cd = CapturedDecode(q0, k, v, splits=8, sharded=sharded)
    kh, vh = k.float().cpu().numpy(), v.float().cpu().numpy()
    for _ in range(2):  # two different queries through the same graph
        q = torch.randn(2, 32, 1, 128, device="cuda", generator=g).to(torch.bfloat16)
        O, L = cd(q)
        torch.cuda.synchronize()
        Or, Lr = ora.decode(q[:, :, 0].float().cpu().numpy(), kh, vh)
        assert_parity(O[:, :, 0], L[:, :, 0], Or, Lr, "bfloat16", 1.0, "graph replay")
        if sharded:
            Oe, Le = decode_kv_sharded(q, k, v, splits=8)
        else:
            Oe, Le = b200attn.decode(q, k, v, splits=8)
        assert torch.equal(O, Oe) and torch.equal(L, Le)
