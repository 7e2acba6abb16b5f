"""The C ABI driven from C: tests/c_host/mm_host.c is built with gcc against
include/tilec_mm.h, the in-tree libtilec_mm.so and the CUDA runtime, the way a cgo / JNI /
N-API host would bind it.  On CPU the program must compile and link; on a B200 it runs
seven products (AUTO split-K, CTA pair, unaligned rows, ragged 3XTF32, TF32, SIMT, and the
allocation-free split-K entry point) and checks each against its own fp64 sums."""
import os
import shutil
import subprocess

import pytest

from tilec_b200 import build

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "c_host", "mm_host.c")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _build_host(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lib = build.build()
    libdir = os.path.dirname(lib)
    exe = str(tmp_path / "mm_host")
    cmd = [cc, "-O2", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), SRC, "-o", exe, "-L", libdir, "-ltilec_mm",
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-lm",
           f"-Wl,-rpath,{libdir}", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_c_host_compiles_and_links(tmp_path):
    assert os.access(_build_host(tmp_path), os.X_OK)


@pytest.mark.gpu
def test_c_host_runs_products_on_gpu(tmp_path):
    exe = _build_host(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL OK" in r.stdout
