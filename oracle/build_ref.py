"""Build the reference's headline kernel for sm_100a into oracle/_ref/ -- TEST
INFRASTRUCTURE ONLY (a parity checker and a measured bar, never shipped).

Compiles the UNMODIFIED reference source cuda/flash_attn_fa3_db_full.cu (the
kernel fa3db_full_fwd_kernel and its pybind module `forward` / `forward_only`)
as a torch extension, with the reference's own flags (setup.py:10-16: -O3
--use_fast_math) except the architecture: -gencode arch=compute_100a,code=sm_100a
instead of sm_89 (an sm_89 cubin does not load on a B200).  Only the source
file is read from the reference checkout; its setup.py is not run.  Output:
oracle/_ref/flash_attn_fa3_db_full.so (git-ignored; it travels to the GPU box).

    python oracle/build_ref.py /path/to/reference   (or B2A_REFERENCE_ROOT=...)
"""
from __future__ import annotations

import glob
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "flash_attn_fa3_db_full"


def so_path() -> str:
    return os.path.join(OUT, NAME + ".so")


def build(ref_root: str) -> str:
    src = os.path.join(ref_root, "cuda", "flash_attn_fa3_db_full.cu")
    if not os.path.exists(src):
        raise FileNotFoundError(src)
    from torch.utils.cpp_extension import load
    bdir = os.path.join(OUT, "build")
    os.makedirs(bdir, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    load(name=NAME, sources=[src], build_directory=bdir, verbose=False,
         extra_cuda_cflags=["-O3", "--use_fast_math",
                            "-gencode", "arch=compute_100a,code=sm_100a"])
    built = glob.glob(os.path.join(bdir, NAME + "*.so"))[0]
    shutil.copy2(built, so_path())
    return so_path()


def load_built():
    """Import the prebuilt module (torch must be importable); None if absent."""
    import importlib.machinery
    import importlib.util
    import torch  # noqa: F401  (the extension links against torch's libraries)
    p = so_path()
    if not os.path.exists(p):
        return None
    loader = importlib.machinery.ExtensionFileLoader(NAME, p)
    spec = importlib.util.spec_from_file_location(NAME, p, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("B2A_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: build_ref.py <reference checkout> (or set B2A_REFERENCE_ROOT)")
    print(build(root))
