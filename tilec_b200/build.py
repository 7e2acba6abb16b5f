"""Build the sm_100a kernel library in-tree: tilec_b200/_lib/libtilec_mm.so.

nvcc cross-compiles for sm_100a without a GPU, so this runs on CPU-only hosts too.
The library is one translation unit (csrc/tilec_mm.cu) exporting the C ABI declared in
include/tilec_mm.h.  Beside it, gcc builds the small CPython module _tilec_fast
(csrc/fastcall.c) through which the Python binding makes its per-call C ABI calls.
Usage: ``python -m tilec_b200.build [--force]``.
"""
import os
import shutil
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB_DIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIB_DIR, "libtilec_mm.so")
HEADER = os.path.join(ROOT, "include", "tilec_mm.h")
FAST_SRC = os.path.join(CSRC, "fastcall.c")
FAST = os.path.join(LIB_DIR, "_tilec_fast" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-shared",
]


def _sources():
    out = [HEADER]
    for f in sorted(os.listdir(CSRC)):
        if f.endswith((".cu", ".cuh", ".h")):
            out.append(os.path.join(CSRC, f))
    return out


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the sm_100a kernel library cannot be built")
    return path


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= t for s in _sources())


def build(force=False, verbose=False):
    """Compile csrc/tilec_mm.cu for sm_100a into _lib/libtilec_mm.so (skipped when fresh)."""
    if not force and up_to_date():
        return LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-o", tmp, os.path.join(CSRC, "tilec_mm.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def fast_up_to_date():
    if not os.path.exists(FAST):
        return False
    t = os.path.getmtime(FAST)
    return all(os.path.getmtime(s) <= t for s in (FAST_SRC, HEADER))


def build_fast(force=False):
    """Compile csrc/fastcall.c into _lib/_tilec_fast (skipped when fresh)."""
    if not force and fast_up_to_date():
        return FAST
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler: the CPython fast-call module cannot be built")
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = FAST + ".tmp"
    cmd = [cc, "-O2", "-shared", "-fPIC", "-std=c11", "-Wall", "-Werror",
           "-I", sysconfig.get_paths()["include"], "-o", tmp, FAST_SRC]
    subprocess.run(cmd, check=True)
    os.replace(tmp, FAST)
    return FAST


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    build_fast(force="--force" in sys.argv)
    print(LIB)
    print(FAST)
