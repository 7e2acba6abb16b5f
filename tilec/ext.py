"""tilec.ext with the reference's names (tilec/ext.py), backed by tilec_b200.ext.

matrix_mul(x1, x2) and _matrix_mul_tiled(x1, x2, BM=64, BN=64, BK=16) run the sm_100a
kernels; cdiv, MAX_BLOCK, plan(N, block=None), mm_configs(M1, N, M2) and the SPLITS /
JOINS / BLOCKS tables return what the reference's return (tilec/ext.py:3,10,29-51).
"""
from tilec_b200.ext import (  # noqa: F401
    BLOCKS,
    JOINS,
    MAX_BLOCK,
    SPLITS,
    _matrix_mul_tiled,
    cdiv,
    check_device,
    matrix_mul,
    mm_configs,
    plan,
)

__all__ = ["matrix_mul", "cdiv", "MAX_BLOCK", "plan", "mm_configs", "SPLITS", "JOINS", "BLOCKS", "check_device"]
