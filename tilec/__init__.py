"""tilec: the reference package name, served by the B200 build (tilec_b200).

Code written against the reference keeps its imports and calls:

    import tilec
    out = tilec.ext.matrix_mul(x1, x2)      # x1 [M, K], x2 [K, N] float32 CUDA tensors

``tilec.ext`` and ``tilec.language`` are the modules of the same names in the reference
(tilec/__init__.py:6-9), restricted to the matrix_mul path: the op, its tiled entry point
and the module-level host helpers (``cdiv``, ``MAX_BLOCK``, ``plan``, ``mm_configs``) with
the reference's signatures and results.  The reference's tile-language compiler (``jit``,
``CompileError``, the Rust/MLIR/Metal toolchain) has no counterpart: the B200 kernels are
built ahead of time, so nothing is compiled at run time.
"""
from . import ext, language  # noqa: F401
from tilec_b200 import TilecError  # noqa: F401

__all__ = ["ext", "language", "TilecError"]
__version__ = "0.1.0"
