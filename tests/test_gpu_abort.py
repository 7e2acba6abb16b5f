"""A GEMM that gives up is visible: NaN where it did not finish, and an error on request.

Failure detection without a fault.  tilec_mm_set_wait_limit shortens every bounded wait
of the library's kernels to 1 ns, so a real GEMM launch gives up at its first wait that
does not pass at once (a copy still in flight, an MMA still running).  Each kernel then
lets its own copies and MMAs land, writes NaN over the output tiles it owns (C, a split-K
slab or a stream-K partial) and returns; the status word reads TILEC_DEV_STATUS_TIMEOUT.
The test checks, for every kernel family, that
  * with TILEC_MM_CHECK=1 the call raises TilecError (the status word, read and cleared);
  * no element of C is left silently wrong: each is NaN or the product's value (within the
    variant's gate), so a poisoned slab reaches C through the split-K reduction;
  * after the limit is restored, the same context computes the product correctly.
No trap, no fault, no endless wait: the context stays usable throughout.
"""
import contextlib
import ctypes

import pytest
import torch

from tilec_b200 import TilecError, _native, ext

pytestmark = pytest.mark.gpu

TOL = {"simt": 1e-5, "splitk": 1e-5, "3xtf32": 1e-5, "3xmixed": 1e-5, "tf32": 5e-3}

# (variant, (M, K, N), split_k, stream_k): the kernel each case reaches.  The tensor-core
# kernels always meet a wait that does not pass at once (the MMA waits for the first
# copies), so they must give up.  The SIMT kernel's only wait is for a B tile whose TMA copy
# was issued three stages earlier and has landed by then, so it may finish: its cases accept
# either outcome, a correct product or the visible give-up.
MAY_FINISH = {"simt", "splitk"}
CASES = [
    ("3xtf32", (512, 4096, 64), 0, False),      # 1-CTA 3xTF32, split-K slabs + reduction
    ("tf32", (512, 4096, 128), 4, False),       # 1-CTA TF32, split-K
    ("3xtf32", (200, 1024, 256), 1, False),     # 1-CTA 3xTF32, BN 256, one slice
    ("3xtf32", (2048, 2048, 2048), 1, False),   # CTA pair, one pair per tile
    ("tf32", (2048, 2048, 2048), 1, False),     # CTA pair, TF32
    ("tf32", (2304, 1024, 2304), 1, False),     # persistent TF32 pairs (81 tiles over the resident pairs)
    ("3xmixed", (2048, 2048, 2048), 1, False),  # CTA pair, mixed split
    ("3xtf32", (1024, 4096, 1024), 3, False),   # CTA pair, split-K
    ("3xtf32", (2304, 2048, 2304), 1, True),    # stream-K pairs with partial tiles
    ("simt", (1024, 2048, 1024), 1, False),     # SIMT with TMA-staged B
    ("splitk", (512, 4096, 64), 0, False),      # SIMT split-K
]


def _status():
    st = ctypes.c_int32(-1)
    _native.check(_native.load().tilec_mm_device_status(None, ctypes.byref(st)), "tilec_mm_device_status")
    return st.value


@contextlib.contextmanager
def _wait_limit(ns):
    lib = _native.load()
    _native.check(lib.tilec_mm_set_wait_limit(ns, None), "tilec_mm_set_wait_limit")
    try:
        yield
    finally:
        _native.check(lib.tilec_mm_set_wait_limit(0, None), "tilec_mm_set_wait_limit")


def _inputs(m, k, n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(m, k, device="cuda", generator=g), torch.randn(k, n, device="cuda", generator=g)


@pytest.mark.parametrize("variant,shape,split_k,stream_k", CASES,
                         ids=[f"{v}-{'x'.join(map(str, s))}-s{k}{'-sk' if sk else ''}" for v, s, k, sk in CASES])
def test_gave_up_is_nan_and_raises_then_context_works(variant, shape, split_k, stream_k, monkeypatch):
    m, k, n = shape
    x1, x2 = _inputs(m, k, n, m + k + n)
    ref = x1.double() @ x2.double()
    assert _status() == 0
    if stream_k:
        assert ext.kernel_plan(x1, x2, variant=variant, stream_k=True, detail=True)["stream_k"]
    out = torch.full((m, n), 12345.0, device="cuda")  # a value no path may leave behind
    monkeypatch.setenv("TILEC_MM_CHECK", "1")
    raised = False
    with _wait_limit(1):
        try:
            ext._matrix_mul(x1, x2, variant=variant, split_k=split_k, out=out, stream_k=stream_k)
        except TilecError as e:
            assert "TIMEOUT" in str(e)
            raised = True
    assert raised or variant in MAY_FINISH, "a tensor-core kernel did not give up at a 1 ns limit"
    assert _status() == 0  # the raising check read and cleared the word (or nothing was set)
    bad = torch.isnan(out)
    assert bad.any() == raised, "NaN without a recorded give-up, or a give-up that left no NaN"
    done = ~bad
    if done.any():
        err = ((out.double() - ref)[done].norm() / ref[done].norm()).item()
        assert err <= TOL[variant], f"finished elements off by {err:.3e}"
    # Limit restored: the same context computes the product, and the check passes.
    out2 = ext._matrix_mul(x1, x2, variant=variant, split_k=split_k, stream_k=stream_k)
    torch.cuda.synchronize()
    err = ((out2.double() - ref).norm() / ref.norm()).item()
    assert torch.isfinite(out2).all() and err <= TOL[variant], err
    assert _status() == 0


def test_check_is_off_by_default_and_status_is_readable(monkeypatch):
    monkeypatch.delenv("TILEC_MM_CHECK", raising=False)
    x1, x2 = _inputs(512, 4096, 64, 3)
    with _wait_limit(1):
        out = ext._matrix_mul(x1, x2, variant="3xtf32")  # returns without raising
        torch.cuda.synchronize()
    assert torch.isnan(out).any()
    with pytest.raises(TilecError, match="TIMEOUT"):
        ext.check_device()
    assert ext.check_device() == 0
