"""Generate tests/golden/golden.npz by running the REFERENCE'S OWN kernel text.

The reference (Naaz30/tilec) cannot run in this container: its compiler needs a Rust
toolchain and MLIR, and its kernels need an Apple GPU.  Its test oracle is torch's
``x1 @ x2`` (tests/test_matmul.py:40) and it ships no golden vectors.  To pin the CPU
oracle to the reference's algorithm anyway, this script

  1. reads tilec/ext.py from a reference checkout (argument or $TILEC_REFERENCE),
  2. extracts only the ``_matmul_tiled`` function definition (ext.py:13-24) with ``ast``
     and drops its ``@jit`` decorator,
  3. executes that function body for every program id of the reference's launch grid
     (cdiv(M, 64), cdiv(N, 64)) with BM=BN=64, BK=16 (ext.py:54,62), under a numpy model
     of the tile-language builtins it uses:
       program_id(axis)      -> the program coordinate
       arange(lo, hi)        -> int64 vector
       zeros(shape)          -> float32 zeros
       load(ptr, mask, other)-> masked gather, `other` where masked off
       store(ptr, val, mask) -> masked scatter
       dot(x, y)             -> float32 matrix product of two 2-D tiles
     and pointer arithmetic ``ptr + offsets`` on the kernel's buffer arguments,
  4. stores the outputs with the SHA-256 of the seeded inputs (tests/golden/gen.py).

Usage:  python tests/golden/make_golden.py /path/to/tilec-checkout
Only this script reads the reference; the tests read the committed golden.npz.
"""
import ast
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import gen  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")


class Ptr:
    """A buffer plus an int64 offset array (the value of `a + rm[:, None] * K + ...`)."""

    def __init__(self, buf, off=0):
        self.buf = buf
        self.off = np.asarray(off, dtype=np.int64)

    def __add__(self, other):
        return Ptr(self.buf, self.off + np.asarray(other, dtype=np.int64))

    __radd__ = __add__


class TileLanguage:
    """numpy semantics of the tilec builtins used by _matmul_tiled (tilec/language.py:13-14)."""

    class constexpr:  # annotation marker only (tilec/language.py:1-3)
        pass

    def __init__(self):
        self.pid = (0, 0, 0)

    def program_id(self, axis):
        return int(self.pid[axis])

    def arange(self, lo, hi):
        return np.arange(lo, hi, dtype=np.int64)

    def zeros(self, shape):
        return np.zeros(shape, dtype=np.float32)

    def load(self, ptr, mask=None, other=0.0):
        off = ptr.off
        if mask is None:
            return ptr.buf[off].astype(np.float32)
        mask = np.broadcast_to(mask, off.shape)
        safe = np.where(mask, off, 0)  # never index out of range (the reference clamps too)
        vals = ptr.buf[safe] if ptr.buf.size else np.zeros(off.shape, np.float32)
        return np.where(mask, vals, np.float32(other)).astype(np.float32)

    def store(self, ptr, val, mask=None):
        off = ptr.off
        val = np.broadcast_to(np.asarray(val, dtype=np.float32), off.shape)
        if mask is None:
            ptr.buf[off] = val
        else:
            mask = np.broadcast_to(mask, off.shape)
            ptr.buf[off[mask]] = val[mask]

    def dot(self, x, y):
        return np.matmul(x.astype(np.float32), y.astype(np.float32)).astype(np.float32)


def load_reference_kernel(ref_root):
    src_path = os.path.join(ref_root, "tilec", "ext.py")
    with open(src_path) as f:
        tree = ast.parse(f.read(), filename=src_path)
    fdef = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "_matmul_tiled")
    fdef.decorator_list = []
    tl = TileLanguage()
    ns = {"tl": tl, "range": range}
    exec(compile(ast.Module(body=[fdef], type_ignores=[]), src_path, "exec"), ns)
    return ns["_matmul_tiled"], tl, (fdef.lineno, fdef.end_lineno)


def run_reference(kernel, tl, x1, x2, BM=64, BN=64, BK=16):
    M, K = x1.shape
    _, N = x2.shape
    a = np.ascontiguousarray(x1).reshape(-1)
    b = np.ascontiguousarray(x2).reshape(-1)
    c = np.full(M * N, np.nan, dtype=np.float32)  # poisoned: every in-range element must be stored
    for p0 in range((M + BM - 1) // BM):
        for p1 in range((N + BN - 1) // BN):
            tl.pid = (p0, p1, 0)
            kernel(Ptr(a), Ptr(b), Ptr(c), M, N, K, BM=BM, BN=BN, BK=BK)
    return c.reshape(M, N)


RANDN_CASES = [(m, k, n, 1000 + i) for i, (m, k, n) in enumerate(gen.REF_TEST_SHAPES)]
EXACT_CASES = [(1, 1, 1, 7), (5, 7, 3, 8), (65, 17, 63, 9), (128, 300, 130, 10), (129, 64, 257, 11),
               (3, 1000, 5, 12)]
SAMPLE_ROWS_ABOVE = 40000  # store a row sample instead of the whole output above this many elements


def main(ref_root):
    kernel, tl, (l0, l1) = load_reference_kernel(ref_root)
    out = {"source": np.array(f"tilec/ext.py:{l0}-{l1} _matmul_tiled, grid (cdiv(M,64),cdiv(N,64)), BK=16")}
    for tag, cases, make in (("randn", RANDN_CASES, gen.randn_inputs), ("exact", EXACT_CASES, gen.exact_inputs)):
        for (m, k, n, seed) in cases:
            x1, x2 = make(m, k, n, seed)
            c = run_reference(kernel, tl, x1, x2)
            assert not np.isnan(c).any(), "reference kernel left an output unwritten"
            key = f"{tag}_{m}x{k}x{n}_s{seed}"
            out[key + "_digest"] = np.array(gen.digest(x1, x2))
            if c.size > SAMPLE_ROWS_ABOVE:
                rows = np.arange(0, m, 17)
                out[key + "_rows"] = rows
                out[key + "_c_rows"] = c[rows]
                out[key + "_rowsum"] = c.astype(np.float64).sum(axis=1)
                out[key + "_colsum"] = c.astype(np.float64).sum(axis=0)
            else:
                out[key + "_c"] = c
            print(key, c.shape)
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ["TILEC_REFERENCE"])
