"""b200attn -- B200-native (sm_100a) attention: prefill forward (O + logsumexp L),
split-KV / paged GQA decode with an LSE-weighted combine, and KV-sharded decode
over NCCL.  A drop-in for the extension modules of Bias92/flashattn-cuda
(`forward(Q, K, V) -> [O, L]`, `forward_only(Q, K, V) -> O`).
"""
from .attention import (backward, check_device, decode, decode_combine, decode_combine_ranks,
                        decode_merge_splits,
                        decode_paged, decode_splitkv, default_scale, device_error_flags, forward,
                        forward_only, forward_varlen)
from ._lib import lib_path

__all__ = ["forward", "forward_only", "forward_varlen", "backward", "decode", "decode_splitkv", "decode_combine",
           "decode_combine_ranks", "decode_merge_splits", "decode_paged", "device_error_flags", "check_device", "default_scale", "lib_path"]
__version__ = "0.1.0"
