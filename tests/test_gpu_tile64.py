"""64-row tiles of the 1-CTA tensor-core kernel (tcgen05.mma M = 64), on a B200.

The reference kernel's tile is 64 rows (tilec/ext.py:54).  The 1-CTA kernel builds
64-row tiles for products of at most 64 rows, for skinny products that would otherwise
split K over most of the SMs, and on request (tile_m=64).  Checked here against the CPU
oracle (the restated reference kernel) at each variant's gate, on ragged and aligned
shapes, one and several K slices, transposed views, batched 64-row slices, and the raw /
masked hi(x) bit equality that the 128-row kernel also meets.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from tilec_b200 import _native, ext

pytestmark = pytest.mark.gpu

TOL = {"tf32": 5e-3, "3xtf32": 1e-5, "3xtf32_masked": 1e-5}


def _inputs(m, k, n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(m, k, generator=g), torch.randn(k, n, generator=g)


def _check(x1, x2, got, variant):
    want = oracle.mm_tiled(x1.numpy(), x2.numpy())
    err = oracle.rel_frob(got.cpu().numpy(), want)
    assert np.isfinite(got.cpu().numpy()).all() and err <= TOL[variant], f"{variant}: relFrob {err:.3e}"


def _status_clean():
    st = ctypes.c_int32(-1)
    _native.check(_native.load().tilec_mm_device_status(None, ctypes.byref(st)), "device_status")
    return st.value == 0


@pytest.mark.parametrize("variant", ("tf32", "3xtf32", "3xtf32_masked"))
@pytest.mark.parametrize("split_k", (1, 3))
@pytest.mark.parametrize("shape", [(64, 1024, 64), (1, 4096, 128), (50, 300, 100), (33, 17, 65), (64, 64, 64),
                                   (512, 4096, 64), (200, 1000, 300), (129, 2048, 130)])
def test_tile64_matches_oracle(shape, split_k, variant):
    m, k, n = shape
    x1, x2 = _inputs(m, k, n, m * 7 + k + n)
    d1, d2 = x1.cuda(), x2.cuda()
    info = ext.kernel_plan(d1, d2, variant=variant, split_k=split_k, tile_m=64, detail=True)
    assert info["tile_m"] == 64, info
    got = ext._matrix_mul(d1, d2, variant=variant, split_k=split_k, tile_m=64)
    _check(x1, x2, got, variant)
    assert _status_clean()


@pytest.mark.parametrize("shape", [(64, 1024, 64), (50, 300, 100), (512, 4096, 64)])
def test_tile64_raw_hi_equals_masked_hi(shape):
    m, k, n = shape
    x1, x2 = _inputs(m, k, n, 3)
    d1, d2 = x1.cuda(), x2.cuda()
    a = ext._matrix_mul(d1, d2, variant="3xtf32", tile_m=64)
    b = ext._matrix_mul(d1, d2, variant="3xtf32_masked", tile_m=64)
    assert torch.equal(a, b)


def test_tile64_is_auto_choice_for_short_and_skinny_products():
    def plan(m, k, n):
        return ext.kernel_plan(torch.empty(m, k, device="cuda"), torch.empty(k, n, device="cuda"), variant="3xtf32",
                               detail=True)
    assert plan(64, 4096, 4096)["tile_m"] == 64
    assert plan(1, 8192, 512)["tile_m"] == 64
    assert plan(512, 4096, 64)["tile_m"] == 128         # config 1: 128-row tiles measured faster
    assert plan(2048, 2048, 2048)["tile_m"] is None      # CTA pair
    assert plan(8192, 1024, 128)["tile_m"] == 128
    # asking for 128-row tiles keeps them
    d = torch.empty(64, 512, device="cuda")
    assert ext.kernel_plan(d, d.t(), variant="3xtf32", tile_m=128, detail=True)["tile_m"] == 128


@pytest.mark.parametrize("variant", ("tf32", "3xtf32"))
@pytest.mark.parametrize("ta,tb", [(False, True), (True, False), (True, True)])
def test_tile64_transposed_views(ta, tb, variant):
    m, k, n = 60, 700, 96
    x1, x2 = _inputs(m, k, n, 9)
    d1 = x1.cuda().t().contiguous().t() if ta else x1.cuda()
    d2 = x2.cuda().t().contiguous().t() if tb else x2.cuda()
    got = ext._matrix_mul(d1, d2, variant=variant, tile_m=64)
    _check(x1, x2, got, variant)


@pytest.mark.parametrize("variant", ("tf32", "3xtf32"))
def test_tile64_batched_64_row_slices(variant):
    """512 products of 64 x 1024 x 64 in one call, the batched case 64-row tiles are for."""
    g = torch.Generator(device="cuda").manual_seed(4)
    a = torch.randn(512, 64, 1024, device="cuda", generator=g)
    b = torch.randn(512, 1024, 64, device="cuda", generator=g)
    got = ext.matrix_mul_ex(a, b, variant=variant)
    ref = torch.bmm(a.double(), b.double())
    err = ((got.double() - ref).norm() / ref.norm()).item()
    assert err <= TOL[variant], err
    # The batched call runs one K slice per product (512 tiles fill the GPU); the same slice
    # alone, asked for one K slice too, gives the same bits.
    assert ext.kernel_plan(a[0], b[0], variant=variant, split_k=1, detail=True)["tile_m"] == 64
    one = ext._matrix_mul(a[77], b[77], variant=variant, split_k=1)
    assert torch.equal(one, got[77])
