"""Build libb200attn.so in-tree with nvcc for sm_100a.

The library is plain CUDA C++ behind the extern "C" ABI of include/b200attn.h;
no torch headers are involved, so a build takes seconds per translation unit
and runs on a machine without a GPU (nvcc cross-compiles).  The reference
builds one torch extension per kernel with setup.py
(setup.py:1-81, `-gencode=arch=compute_89,code=sm_89`); this replaces that step.

Usage:  python -m b200attn.build [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)                      # flashattn-cuda_b200/
CSRC = os.path.join(ROOT, "csrc")
BUILD_DIR = os.path.join(ROOT, "_build")
INCLUDE = os.path.join(os.path.dirname(ROOT), "include")
LIB_PATH = os.path.join(PKG_DIR, "libb200attn.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the b200attn CUDA library cannot be built")
    return cand


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _fastcall_path() -> str:
    import sysconfig
    return os.path.join(PKG_DIR, "_fastcall" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_fastcall(force: bool = False, verbose: bool = False) -> str | None:
    """Compile the CPython binding csrc/fastcall.c against libb200attn.so (rpath
    $ORIGIN).  Returns its path, or None when no C compiler / Python headers exist
    (the package then calls the library through ctypes only)."""
    import sysconfig
    src = os.path.join(CSRC, "fastcall.c")
    out = _fastcall_path()
    inc = sysconfig.get_paths()["include"]
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None or not os.path.exists(os.path.join(inc, "Python.h")):
        return None
    if not force and not _stale(out, [src, LIB_PATH, os.path.join(INCLUDE, "b200attn.h")]):
        return out
    cmd = [cc, "-O2", "-shared", "-fPIC", "-I", inc, src, "-o", out + ".tmp", "-L", PKG_DIR,
           "-l:libb200attn.so", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"fastcall build failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(out + ".tmp", out)
    return out


def _deps() -> list[str]:
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hdrs.append(os.path.join(INCLUDE, "b200attn.h"))
    return hdrs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every csrc/*.cu for sm_100a and link libb200attn.so; returns its path."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    nvcc = _nvcc()
    hdrs = _deps()
    jobs = []
    objs = []
    for src in _sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            cmd = [nvcc, *NVCC_FLAGS, *ARCH_FLAGS, "-I", INCLUDE, "-c", src, "-o", obj]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(run, jobs))
    if force or jobs or _stale(LIB_PATH, objs):
        tmp = LIB_PATH + ".tmp"
        run([nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", tmp, *objs])
        os.replace(tmp, LIB_PATH)
    build_fastcall(force=force, verbose=verbose)
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)
