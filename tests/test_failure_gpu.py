"""Failure detection on the device, exercised without a GPU fault.

Every pipeline wait in the library is bounded: one that is never satisfied
gives up after its limit, records bit 0 of the device error word and lets the
CTA wind down, and the host sees B2A_ERR_TIMEOUT.  b2a_selftest_wait_timeout
makes one such wait run out on purpose (a single thread waiting ~1 ms on an
mbarrier nothing arrives at, with no copy or tensor-core work in flight), so
the test checks the status and that the device still answers afterwards.  The
reference has host checks only (cuda/flash_attn_fa3_db_full.cu:352-363, :399).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_parity
from oracle import attention as ora

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_device_stays_usable():
    import b200attn
    from b200attn import _lib
    lib = _lib.load()
    b200attn.device_error_flags()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        rc = lib.b2a_selftest_wait_timeout(1000, stream)
        assert rc == _lib.B2A_ERR_TIMEOUT, lib.b2a_last_error()
        assert b"gave up" in lib.b2a_last_error()
    # the self-test consumed its own flag: the shared word reads clean
    assert b200attn.device_error_flags() == 0
    # and the device answers: a small forward still matches the oracle
    q = torch.from_numpy(ora.seeded_normal((1, 2, 200, 64), 1)).half().cuda()
    k = torch.from_numpy(ora.seeded_normal((1, 2, 200, 64), 2)).half().cuda()
    v = torch.from_numpy(ora.seeded_normal((1, 2, 200, 64), 3)).half().cuda()
    O, L = b200attn.forward(q, k, v)
    Or, Lr = ora.naive_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                 v.float().cpu().numpy())
    assert_parity(O, L, Or, Lr, "float16")
    assert b200attn.device_error_flags() == 0
