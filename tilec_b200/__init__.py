"""tilec_b200: B200-native (sm_100a) implementation of tilec's one op, ``ext.matrix_mul``.

    import torch, tilec_b200
    x1 = torch.randn(512, 4096, device="cuda")
    x2 = torch.randn(4096, 64, device="cuda")
    out = tilec_b200.ext.matrix_mul(x1, x2)

Layout: ``ext`` (the drop-in op, tilec/ext.py), ``language`` (host helpers), ``select``
(per-shape kernel selection, the B200 counterpart of tilec/tune.py), ``dist`` (row-
sharded multi-GPU matrix_mul over NCCL), ``_native`` (ctypes binding of the C ABI in
include/tilec_mm.h), ``build`` (nvcc build of the in-tree kernel library).
Importing the package needs no GPU and no compiler; the kernel library is loaded on
first use.
"""
from . import ext, language  # noqa: F401
from ._native import TilecError  # noqa: F401

__all__ = ["ext", "language", "TilecError"]
__version__ = "0.1.0"
