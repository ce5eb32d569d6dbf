"""C-ABI boundary checks that need no GPU: libb200attn.so loads, exports every
function include/b200attn.h declares, and the Python mirror of the reference's
module rejects bad inputs with the reference's messages
(cuda/flash_attn_fa3_db_full.cu:352-363) before touching a device."""
from __future__ import annotations

import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "b200attn.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2a_\w+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ("b2a_prefill_fwd", "b2a_decode_splitkv", "b2a_decode_combine",
              "b2a_decode_paged", "b2a_status_string", "b2a_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from b200attn import _lib
    lib = ctypes.CDLL(_lib.lib_path())
    for name in declared_functions():
        assert hasattr(lib, name), name
    # and the Python binding declares a signature for each one
    assert set(declared_functions()) <= set(_lib.EXPORTED)


def test_status_strings_and_version():
    from b200attn import _lib
    lib = _lib.load()
    assert lib.b2a_status_string(0) == b"ok"
    assert lib.b2a_status_string(3) == b"misaligned pointer"
    assert lib.b2a_version() == b"0.1.0"


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU failure path")
def test_no_device_is_reported_not_faulted():
    from b200attn import _lib
    lib = _lib.load()
    rc = lib.b2a_prefill_fwd(None, None, None, None, None, 1, 1, 1, 64, 64, 0, 0, 0.125, None)
    assert rc == 6  # B2A_ERR_NO_DEVICE
    assert b"sm_100" in lib.b2a_last_error()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU failure path")
def test_fastcall_binding_shares_the_library():
    """The CPython binding calls the same loaded libb200attn.so as ctypes: an
    error it triggers is visible through the ctypes handle's b2a_last_error."""
    from b200attn import _lib
    import b200attn.attention as A
    if A._fastcall is None:
        pytest.skip("CPython binding not built")
    lib = _lib.load()
    lib.b2a_status_string(0)
    rc = A._fastcall.prefill_fwd_kv(0, 0, 0, 0, 0, 1, 1, 1, 64, 64, 64, 0, 0, 0.125, 0)
    assert rc == 6  # B2A_ERR_NO_DEVICE
    assert b"sm_100" in lib.b2a_last_error()


def test_python_api_rejects_like_the_reference():
    import b200attn
    q = torch.zeros(1, 1, 8, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="must be CUDA tensors"):
        b200attn.forward(q, q, q)
    with pytest.raises(RuntimeError, match="must be CUDA tensors"):
        b200attn.forward_only(q, q, q)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        b200attn.decode(q[:, :, 0], q, q)


def test_selftest_rejects_bad_limit():
    from b200attn import _lib
    lib = _lib.load()
    assert lib.b2a_selftest_wait_timeout(0, None) == 1
    assert lib.b2a_selftest_wait_timeout(2_000_000, None) == 1


def test_device_error_reports_timeout_status(monkeypatch):
    """(No GPU needed: the library call is faked.)  b2a_device_error returns B2A_ERR_TIMEOUT when bit 0 is set; the Python
    reader returns the flags and check_device() raises."""
    import b200attn
    from b200attn import _lib, attention as A
    lib = _lib.load()

    class FakeLib:
        def b2a_device_error(self, p):
            p._obj.value = 1
            return _lib.B2A_ERR_TIMEOUT

        def __getattr__(self, n):
            return getattr(lib, n)

    monkeypatch.setattr(_lib, "load", lambda: FakeLib())
    assert A.device_error_flags() == 1
    with pytest.raises(RuntimeError, match="wait timed out"):
        A.check_device()
