"""Seeded input generators shared by the golden-fixture script and the tests.

Inputs are regenerated, not stored: each fixture records the SHA-256 of the inputs it
was made from, and the tests check that hash before comparing outputs.
"""
import hashlib

import numpy as np

# The reference test's parametrised shapes (m, k, n): tests/test_matmul.py:33.
REF_TEST_SHAPES = [(1, 1, 1), (5, 7, 3), (65, 17, 63), (128, 300, 130), (512, 1024, 256)]


def randn_inputs(m, k, n, seed):
    """x1 [m,k], x2 [k,n] i.i.d. N(0,1) float32 from numpy's PCG64 stream."""
    g = np.random.Generator(np.random.PCG64(seed))
    x1 = g.standard_normal((m, k), dtype=np.float32)
    x2 = g.standard_normal((k, n), dtype=np.float32)
    return x1, x2


def exact_inputs(m, k, n, seed):
    """Operands j/8 with integer j in [-8, 8].

    Every product is a multiple of 1/64 with |p| <= 1, so any partial sum of up to 2^18
    terms is an exact fp32 value: every correct summation order -- and TF32 tensor
    cores, whose 10-bit mantissa holds these operands exactly -- yields the same bits.
    """
    g = np.random.Generator(np.random.PCG64(seed))
    x1 = (g.integers(-8, 9, size=(m, k)).astype(np.float32) / np.float32(8))
    x2 = (g.integers(-8, 9, size=(k, n)).astype(np.float32) / np.float32(8))
    return x1, x2


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def config4_shapes(n=64, seed=4):
    """Benchmark config 4: seeded log-uniform (M, K, N) triples over [1, 8192]^3.

    Modelled on the reference tuner's shape sampler (tilec/tune.py:54-65) but spanning
    [1, 8192] per dimension; the first triple is forced to M = 1 (GEMV-like) and the
    second to N <= 64 (skinny), so both cases are always present.
    """
    import random
    rng = random.Random(seed)
    out = []
    seen = set()
    while len(out) < n:
        m, k, nn = (max(1, round(2 ** rng.uniform(0, 13))) for _ in range(3))
        if len(out) == 0:
            m = 1
        elif len(out) == 1:
            nn = min(nn, 64)
        if (m, k, nn) in seen:
            continue
        seen.add((m, k, nn))
        out.append((m, k, nn))
    return out


# Benchmark configs 1-3 and 5 as (M, K, N, distribution).
CONFIG1 = (512, 4096, 64, "normal")
CONFIG2 = (2048, 2048, 2048, "normal")
CONFIG3 = (1000, 3001, 777, "uniform")
CONFIG5 = (65536, 8192, 8192, "config5")
