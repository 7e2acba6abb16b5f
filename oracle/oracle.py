"""ctypes/numpy wrappers of the CPU oracle (test infrastructure only; see __init__.py)."""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "_build", "libtilec_oracle.so")
_lib = None


def lib_path():
    return _LIB


def build(force=False):
    """Compile oracle/mm_tiled.c into oracle/_build/libtilec_oracle.so (make)."""
    if force or not os.path.exists(_LIB) or os.path.getmtime(_LIB) < os.path.getmtime(
            os.path.join(_HERE, "mm_tiled.c")):
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "_build/libtilec_oracle.so"],
                       check=True)
    return _LIB


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(_LIB)
        i64 = ctypes.c_int64
        fp = ctypes.c_void_p
        lib.tilec_oracle_mm_tiled.argtypes = [fp, fp, fp, i64, i64, i64, i64, i64, i64,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.tilec_oracle_mm_tiled.restype = ctypes.c_int
        lib.tilec_oracle_mm_f64.argtypes = [fp, fp, fp, i64, i64, i64, i64, i64, i64]
        lib.tilec_oracle_mm_f64.restype = ctypes.c_int
        _lib = lib
    return _lib


def _as_f32(x):
    x = np.asarray(x)
    if x.dtype != np.float32:
        raise TypeError(f"oracle expects float32, got {x.dtype}")
    return np.ascontiguousarray(x)


def mm_tiled(x1, x2, BM=64, BN=64, BK=16):
    """Restated reference kernel (tilec/ext.py:13-24) on numpy fp32 arrays."""
    a, b = _as_f32(x1), _as_f32(x2)
    M, K = a.shape
    K2, N = b.shape
    if K != K2:
        raise ValueError(f"matrix_mul: shapes {a.shape} and {b.shape} don't match")
    c = np.empty((M, N), np.float32)
    if M and N:
        rc = _load().tilec_oracle_mm_tiled(a.ctypes.data, b.ctypes.data, c.ctypes.data, M, N, K,
                                           max(K, 1), max(N, 1), max(N, 1), BM, BN, BK)
        if rc:
            raise RuntimeError("oracle mm_tiled failed")
    return c


def mm_f64(x1, x2):
    """fp64-accumulated product of fp32 operands (returns float64)."""
    a, b = _as_f32(x1), _as_f32(x2)
    M, K = a.shape
    _, N = b.shape
    c = np.empty((M, N), np.float64)
    if M and N:
        rc = _load().tilec_oracle_mm_f64(a.ctypes.data, b.ctypes.data, c.ctypes.data, M, N, K,
                                         max(K, 1), max(N, 1), max(N, 1))
        if rc:
            raise RuntimeError("oracle mm_f64 failed")
    return c


def mm_torch(x1, x2, threads=None):
    """The reference test's oracle expression ``x1 @ x2`` (tests/test_matmul.py:40) in torch fp32 on CPU."""
    import torch
    if threads is not None:
        torch.set_num_threads(threads)
    t1 = torch.as_tensor(np.asarray(x1)) if not isinstance(x1, torch.Tensor) else x1.cpu()
    t2 = torch.as_tensor(np.asarray(x2)) if not isinstance(x2, torch.Tensor) else x2.cpu()
    return (t1.float() @ t2.float()).numpy()


def rel_frob(got, ref):
    """||got - ref||_F / ||ref||_F in float64 (0 when both are zero)."""
    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(r)
    num = np.linalg.norm(g - r)
    if den == 0.0:
        return float(num)
    return float(num / den)
