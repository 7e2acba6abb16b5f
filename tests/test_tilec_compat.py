"""The reference's import path and host helpers: ``import tilec; tilec.ext.matrix_mul``.

CPU tests: the ``tilec`` package imports without a GPU; its host helpers return what the
reference's own helpers return (tests/golden/host_helpers.json, made by executing the
reference's code, tests/golden/make_host_golden.py); the shape error keeps its text.
GPU test: the body of the reference's test_matrix_mul (tests/test_matmul.py:32-40), with
"cuda" in place of "mps", run through ``import tilec``.
"""
import inspect
import json
import os

import numpy as np
import pytest
import torch

import tilec
import tilec.language as tl
from tilec import ext

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "host_helpers.json")


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)


def test_package_surface():
    assert tilec.ext is ext and hasattr(tilec, "language")
    for name in ("matrix_mul", "_matrix_mul_tiled", "cdiv", "MAX_BLOCK", "plan", "mm_configs"):
        assert hasattr(ext, name), name
    assert list(inspect.signature(ext.matrix_mul).parameters) == ["x1", "x2"]
    assert list(inspect.signature(ext.plan).parameters) == ["N", "block"]
    assert inspect.signature(ext.plan).parameters["block"].default is None
    assert list(inspect.signature(ext.mm_configs).parameters) == ["M1", "N", "M2"]
    sig = inspect.signature(ext._matrix_mul_tiled).parameters
    assert [(k, v.default) for k, v in sig.items()][2:] == [("BM", 64), ("BN", 64), ("BK", 16)]
    assert tl.cdiv is ext.cdiv


def test_constants_match_reference(golden):
    assert ext.MAX_BLOCK == golden["MAX_BLOCK"]
    assert list(ext.SPLITS) == golden["SPLITS"]
    assert list(ext.JOINS) == golden["JOINS"]
    assert list(ext.BLOCKS) == golden["BLOCKS"]


def test_cdiv_matches_reference(golden):
    for a, b, want in golden["cdiv"]:
        assert ext.cdiv(a, b) == tl.cdiv(a, b) == want


def test_plan_matches_reference(golden):
    for n, want in golden["plan"]:
        assert list(ext.plan(n)) == want, n
    for n, b, want in golden["plan_block"]:
        assert list(ext.plan(n, b)) == want, (n, b)
        assert list(ext.plan(n, block=b)) == want


def test_mm_configs_matches_reference(golden):
    for args, want in golden["mm_configs"]:
        assert [list(c) for c in ext.mm_configs(*args)] == want, args


def test_shape_error_text():
    with pytest.raises(ValueError, match=r"matrix_mul: shapes \(3, 4\) and \(5, 6\) don't match"):
        ext.matrix_mul(torch.zeros(3, 4), torch.zeros(5, 6))
    with pytest.raises(ValueError):
        ext.matrix_mul(torch.zeros(3), torch.zeros(3, 2))
    with pytest.raises(ValueError):
        ext._matrix_mul_tiled(torch.zeros(2, 2), torch.zeros(2, 2), BM=0)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(1, 1, 1), (5, 7, 3), (65, 17, 63), (128, 300, 130), (512, 1024, 256)])
def test_matrix_mul(shape):
    m, k, n = shape
    x1 = torch.randn(m, k, device="cuda")
    x2 = torch.randn(k, n, device="cuda")
    got = ext.matrix_mul(x1, x2)
    torch.cuda.synchronize()
    np.testing.assert_allclose(got.cpu().numpy(), (x1 @ x2).cpu().numpy(), rtol=1e-3, atol=1e-2)


@pytest.mark.gpu
def test_matrix_mul_tiled_entry_point():
    g = torch.Generator(device="cuda").manual_seed(5)
    x1 = torch.randn(300, 520, device="cuda", generator=g)
    x2 = torch.randn(520, 700, device="cuda", generator=g)
    got = ext._matrix_mul_tiled(x1, x2, BM=64, BN=64, BK=16)
    ref = x1.double() @ x2.double()
    assert ((got.double() - ref).norm() / ref.norm()).item() <= 1e-5
