"""The CPU oracle, pinned against golden vectors made by the reference's own kernel text.

tests/golden/golden.npz was produced by tests/golden/make_golden.py, which executes
``_matmul_tiled`` from tilec/ext.py:13-24 over its launch grid (ext.py:62) under a numpy
model of the tile-language builtins.  The restated oracle (oracle/mm_tiled.c) must
reproduce it bit for bit on exactly representable inputs and to fp32 rounding
(relative Frobenius error <= 1e-6) on N(0,1) inputs.
"""
import numpy as np
import pytest

import gen
import oracle

GOLDEN = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "golden.npz"))


def _cases():
    out = []
    for k in sorted(GOLDEN.files):
        if k.endswith("_digest"):
            base = k[: -len("_digest")]
            tag, shape, s = base.split("_")
            m, kk, n = map(int, shape.split("x"))
            out.append((base, tag, m, kk, n, int(s[1:])))
    return out


CASES = _cases()


def _inputs(tag, m, k, n, seed):
    return (gen.randn_inputs if tag == "randn" else gen.exact_inputs)(m, k, n, seed)


def test_golden_covers_reference_test_shapes():
    shapes = {(m, k, n) for (_, tag, m, k, n, _) in CASES if tag == "randn"}
    assert shapes == set(gen.REF_TEST_SHAPES)
    assert "tilec/ext.py" in str(GOLDEN["source"])


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_oracle_matches_reference_kernel(case):
    base, tag, m, k, n, seed = case
    x1, x2 = _inputs(tag, m, k, n, seed)
    assert gen.digest(x1, x2) == str(GOLDEN[base + "_digest"]), "input generator drifted from the fixture"
    c = oracle.mm_tiled(x1, x2)
    if base + "_c" in GOLDEN.files:
        ref = GOLDEN[base + "_c"]
        got = c
    else:
        rows = GOLDEN[base + "_rows"]
        ref = GOLDEN[base + "_c_rows"]
        got = c[rows]
        np.testing.assert_allclose(c.astype(np.float64).sum(axis=1), GOLDEN[base + "_rowsum"], rtol=1e-5, atol=1e-3)
        np.testing.assert_allclose(c.astype(np.float64).sum(axis=0), GOLDEN[base + "_colsum"], rtol=1e-5, atol=1e-3)
    if tag == "exact":
        assert np.array_equal(got, ref)
    else:
        assert oracle.rel_frob(got, ref) <= 1e-6


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (5, 7, 3), (65, 17, 63), (128, 300, 130), (512, 4096, 64)])
def test_oracle_vs_fp64_and_torch(m, k, n):
    x1, x2 = gen.randn_inputs(m, k, n, 7)
    c = oracle.mm_tiled(x1, x2)
    assert oracle.rel_frob(c, oracle.mm_f64(x1, x2)) <= 1e-6
    assert oracle.rel_frob(oracle.mm_torch(x1, x2), oracle.mm_f64(x1, x2)) <= 1e-6
    np.testing.assert_allclose(c, oracle.mm_torch(x1, x2), rtol=1e-3, atol=1e-2)


def test_oracle_edge_cases():
    # K == 0: accumulator stays zero and is stored (ext.py:18,24).
    c = oracle.mm_tiled(np.zeros((3, 0), np.float32), np.zeros((0, 4), np.float32))
    assert c.shape == (3, 4) and not c.any()
    # M == 0 / N == 0: empty result.
    assert oracle.mm_tiled(np.zeros((0, 5), np.float32), np.zeros((5, 4), np.float32)).shape == (0, 4)
    assert oracle.mm_tiled(np.zeros((3, 5), np.float32), np.zeros((5, 0), np.float32)).shape == (3, 0)
    # Masked edges: every tile size gives the same exact answer.
    x1, x2 = gen.exact_inputs(70, 33, 90, 3)
    ref = oracle.mm_f64(x1, x2)
    for bm, bn, bk in [(64, 64, 16), (1, 1, 1), (128, 32, 8), (7, 5, 3)]:
        assert np.array_equal(oracle.mm_tiled(x1, x2, bm, bn, bk), ref.astype(np.float32))


def test_oracle_rejects_mismatch_and_dtype():
    with pytest.raises(ValueError, match="don't match"):
        oracle.mm_tiled(np.zeros((2, 3), np.float32), np.zeros((4, 2), np.float32))
    with pytest.raises(TypeError):
        oracle.mm_tiled(np.zeros((2, 3)), np.zeros((3, 2)))


def test_planted_mistake_is_caught():
    """A wrong answer planted in the oracle's output must fail the golden comparison."""
    base, tag, m, k, n, seed = next(c for c in CASES if c[1] == "exact" and c[2] > 1)
    x1, x2 = _inputs(tag, m, k, n, seed)
    c = oracle.mm_tiled(x1, x2)
    c[m // 2, n // 2] += np.float32(1.0 / 64)
    assert not np.array_equal(c, GOLDEN[base + "_c"])
