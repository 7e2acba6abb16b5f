"""The allocation-free entry point tilec_mm_f32_splitk_noalloc, through the C ABI (GPU).

It serves callers that may not allocate device memory (an FFI host that binds only the
C ABI and owns no device allocator, or a process that reserves all device memory up
front).  Its split-K partial sums live in a fixed device array inside the library, so
the test checks, on two calls in a row, that it returns what the allocating entry point
(tilec_mm_f32 with a caller-provided workspace, variant SPLITK) returns and what the CPU
oracle (the restated reference kernel, oracle.mm_tiled) returns, within the tolerance
the other parity tests use, and that explicit requests whose slices do not fit are
refused.  This file sorts last so that a run stopping at the first failure has run every
other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from tilec_b200 import _native, ext

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20  # TILEC_MM_NOALLOC_SCRATCH_BYTES in include/tilec_mm.h
TOL = 1e-5                # relative Frobenius error, as for the SIMT/SPLITK parity tests


def _rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm()).item()


def _noalloc(x1, x2, out, split_k=0):
    lib = _native.load()
    M, K = x1.shape
    N = x2.shape[1]
    stream = torch.cuda.current_stream().cuda_stream
    return lib.tilec_mm_f32_splitk_noalloc(x1.data_ptr(), x2.data_ptr(), out.data_ptr(), M, N, K,
                                           x1.stride(0), x2.stride(0), out.stride(0), split_k, stream)


@pytest.mark.parametrize("shape", [(512, 4096, 64), (1000, 3001, 777), (65, 17, 63), (2, 20000, 33)])
def test_noalloc_matches_allocating_entry_point(shape):
    m, k, n = shape
    g = torch.Generator(device="cuda").manual_seed(m + k + n)
    x1 = torch.randn(m, k, device="cuda", generator=g)
    x2 = torch.randn(k, n, device="cuda", generator=g)
    ref = ext._matrix_mul(x1, x2, variant="splitk")
    want = torch.from_numpy(oracle.mm_tiled(x1.cpu().numpy(), x2.cpu().numpy()))
    for _ in range(2):  # two calls in a row: the shared scratch keeps the previous call's sums
        out = torch.full((m, n), float("nan"), device="cuda")
        assert _noalloc(x1, x2, out) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert _rel(out, ref) <= TOL
        assert _rel(out.cpu(), want) <= TOL


def test_noalloc_explicit_split_and_limit():
    m, k, n = 512, 4096, 64
    g = torch.Generator(device="cuda").manual_seed(3)
    x1 = torch.randn(m, k, device="cuda", generator=g)
    x2 = torch.randn(k, n, device="cuda", generator=g)
    ref = ext._matrix_mul(x1, x2, variant="splitk", split_k=8)
    want = torch.from_numpy(oracle.mm_tiled(x1.cpu().numpy(), x2.cpu().numpy()))
    out = torch.empty(m, n, device="cuda")
    assert _noalloc(x1, x2, out, split_k=8) == 0
    torch.cuda.synchronize()
    assert _rel(out, ref) <= TOL
    assert _rel(out.cpu(), want) <= TOL
    # 64 slices of a 4096 x 1024 output need 1 GiB of partial sums: refused, nothing launched.
    big1 = torch.randn(4096, 256, device="cuda", generator=g)
    big2 = torch.randn(256, 1024, device="cuda", generator=g)
    big_out = torch.empty(4096, 1024, device="cuda")
    assert 64 * 4096 * 1024 * 4 > SCRATCH_BYTES
    assert _noalloc(big1, big2, big_out, split_k=64) == 8  # TILEC_ERR_TOO_LARGE
    # library-chosen slicing stays within the scratch and still returns the product
    assert _noalloc(big1, big2, big_out) == 0
    torch.cuda.synchronize()
    assert _rel(big_out, big1.double() @ big2.double()) <= TOL
    st = ctypes.c_int32(-1)
    assert _native.load().tilec_mm_device_status(None, ctypes.byref(st)) == 0 and st.value == 0


def _case(m, k, n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x1 = torch.randn(m, k, device="cuda", generator=g)
    x2 = torch.randn(k, n, device="cuda", generator=g)
    return x1, x2, torch.from_numpy(oracle.mm_tiled(x1.cpu().numpy(), x2.cpu().numpy()))


def test_noalloc_split_above_cap_and_rounded_split():
    # split_k = 100 runs as 64 slices (the cap); 64 x 64 x 64 x 4 bytes fit in the scratch.
    x1, x2, want = _case(64, 4096, 64, 11)
    out = torch.empty(64, 64, device="cuda")
    assert _noalloc(x1, x2, out, split_k=100) == 0
    torch.cuda.synchronize()
    assert _rel(out.cpu(), want) <= TOL
    # K = 33 with split_k = 8 runs as 3 slices of 16-deep K blocks: 3 slabs of 1024 x 1024
    # fit (12 MiB of 16), although 8 would not.
    x1, x2, want = _case(1024, 33, 1024, 12)
    assert 8 * 1024 * 1024 * 4 > SCRATCH_BYTES >= 3 * 1024 * 1024 * 4
    out = torch.empty(1024, 1024, device="cuda")
    for _ in range(2):
        out.fill_(float("nan"))
        assert _noalloc(x1, x2, out, split_k=8) == 0
        torch.cuda.synchronize()
        assert np.isfinite(out.cpu().numpy()).all()
        assert _rel(out.cpu(), want) <= TOL
