"""ctypes binding of libb200attn.so (the extern "C" ABI in include/b200attn.h).

The library is loaded from this package directory only.  If it is missing the
import fails loudly: there is no CPU or eager fallback for any entry point.
"""
from __future__ import annotations

import ctypes
import os

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libb200attn.so")

B2A_OK = 0
B2A_ERR_TIMEOUT = 5
B2A_F16 = 0
B2A_BF16 = 1

_c_int, _c_float, _vp = ctypes.c_int, ctypes.c_float, ctypes.c_void_p

_SIGNATURES = {
    "b2a_status_string": (ctypes.c_char_p, [_c_int]),
    "b2a_last_error": (ctypes.c_char_p, []),
    "b2a_version": (ctypes.c_char_p, []),
    # q k v o lse | B H Hkv N D | dtype causal scale stream
    "b2a_prefill_fwd": (_c_int, [_vp, _vp, _vp, _vp, _vp] + [_c_int] * 5
                        + [_c_int, _c_int, _c_float, _vp]),
    # q k v o lse | B H Hkv N Nk D | dtype causal scale stream
    "b2a_prefill_fwd_kv": (_c_int, [_vp, _vp, _vp, _vp, _vp] + [_c_int] * 6
                           + [_c_int, _c_int, _c_float, _vp]),
    # q k v o lse cu_q cu_k | B H Hkv total_q total_k max_seqlen_q D | dtype causal scale stream
    "b2a_prefill_fwd_varlen": (_c_int, [_vp] * 7 + [_c_int] * 7 + [_c_int, _c_int, _c_float, _vp]),
    # q k v o_part l_part | B H Hkv Lkv D splits | dtype scale stream
    "b2a_decode_splitkv": (_c_int, [_vp] * 5 + [_c_int] * 6 + [_c_int, _c_float, _vp]),
    # o_part l_part o lse | B H splits D dtype | stream
    "b2a_decode_combine": (_c_int, [_vp] * 4 + [_c_int] * 5 + [_vp]),
    "b2a_exchange_bytes": (ctypes.c_int64, [_c_int] * 4),
    "b2a_exchange_alloc": (_c_int, [ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p), _vp]),
    "b2a_exchange_open": (_c_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "b2a_exchange_close": (_c_int, [_vp]),
    "b2a_exchange_free": (_c_int, [_vp]),
    # o_part l_part peers | rank world | o lse | B H splits D dtype | stream
    "b2a_decode_exchange_combine": (_c_int, [_vp] * 3 + [_c_int] * 2 + [_vp] * 2 + [_c_int] * 5
                                    + [_vp]),
    # o_part l_part o_merged l_merged | B H splits D | stream
    "b2a_decode_merge_splits": (_c_int, [_vp] * 4 + [_c_int] * 4 + [_vp]),
    # o_part l_part o lse | B H splits ranks | rank_stride | D dtype | stream
    "b2a_decode_combine_ranks": (_c_int, [_vp] * 4 + [_c_int] * 4 + [ctypes.c_int64]
                                 + [_c_int] * 2 + [_vp]),
    # q kp vp bt lens o_part l_part o lse | B H Hkv D page max_pages num_pages pps | dtype scale stream
    "b2a_decode_paged": (_c_int, [_vp] * 9 + [_c_int] * 8 + [_c_int, _c_float, _vp]),
    # q kp vp bt lens o lse | B H Hkv D page max_pages num_pages pps | dtype scale stream
    "b2a_decode_paged_noalloc": (_c_int, [_vp] * 7 + [_c_int] * 8 + [_c_int, _c_float, _vp]),
    # k_new v_new k_pool v_pool bt lens | B Hkv T D page max_pages num_pages dtype advance | stream
    "b2a_kv_append_paged": (_c_int, [_vp] * 6 + [_c_int] * 9 + [_vp]),
    # q k v o dO lse dq dk dv ws | B H Hkv N Nk D dtype causal | scale stream
    "b2a_backward": (_c_int, [_vp] * 10 + [_c_int] * 8 + [_c_float, _vp]),
    "b2a_backward_workspace_floats": (ctypes.c_int64, [_c_int] * 4),
    "b2a_device_error": (_c_int, [ctypes.POINTER(ctypes.c_uint32)]),
    "b2a_selftest_wait_timeout": (_c_int, [_c_int, _vp]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None


def lib_path() -> str:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load libb200attn.so (once) and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        raise RuntimeError(
            f"b200attn: {_LIB_PATH} is missing; build it with `python -m b200attn.build` "
            "(there is no fallback implementation)")
    lib = ctypes.CDLL(_LIB_PATH)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int) -> None:
    """Raise RuntimeError with the library's message for a non-OK status."""
    if status != B2A_OK:
        lib = load()
        msg = lib.b2a_last_error().decode() or lib.b2a_status_string(status).decode()
        raise RuntimeError(msg)
