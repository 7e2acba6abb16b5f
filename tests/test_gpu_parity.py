"""Parity of every kernel variant against the CPU oracle, on a B200 (run with -m gpu).

Gates (relative Frobenius error against the oracle, fp32 in / fp32 out):
  SIMT, SPLITK, 3XTF32, 3XMIXED : <= 1e-5        TF32 : <= 5e-3
plus the reference test's own check, np.testing.assert_allclose(rtol=1e-3, atol=1e-2)
against ``x1 @ x2`` (tests/test_matmul.py:40), on the reference test's shapes
(tests/test_matmul.py:33).  Exactly representable inputs must match bit for bit.
Large configs are checked through sampled rows against an fp64 product and a
row-checksum identity C.1 = x1.(x2.1) evaluated in fp64.
"""
import ctypes

import numpy as np
import pytest
import torch

import gen
import oracle
from tilec_b200 import TilecError, _native, ext

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TOL = {"simt": 1e-5, "splitk": 1e-5, "3xtf32": 1e-5, "3xtf32_masked": 1e-5, "3xmixed": 1e-5, "tf32": 5e-3,
       "auto": 1e-5}
TENSOR = ("tf32", "3xtf32", "3xtf32_masked", "3xmixed")
SK_VARIANTS = ("tf32", "3xtf32", "3xtf32_masked")  # variants with a stream-K form
ALL = ("auto", "simt", "splitk", "tf32", "3xtf32", "3xtf32_masked", "3xmixed")


def _aligned(k, n):
    return k % 4 == 0 and n % 4 == 0


def _run(x1, x2, variant, split_k=0):
    d1 = torch.as_tensor(x1).to(DEV)
    d2 = torch.as_tensor(x2).to(DEV)
    return ext._matrix_mul(d1, d2, variant=variant, split_k=split_k).cpu().numpy()


def _status_clean():
    st = ctypes.c_int32(-1)
    _native.check(_native.load().tilec_mm_device_status(None, ctypes.byref(st)), "device_status")
    return st.value == 0


@pytest.mark.parametrize("variant", ALL)
@pytest.mark.parametrize("shape", gen.REF_TEST_SHAPES)
def test_reference_test_shapes(shape, variant):
    m, k, n = shape
    x1, x2 = gen.randn_inputs(m, k, n, 42)
    got = _run(x1, x2, variant)
    if variant != "tf32":
        # The reference test's check (fp32 tolerance); plain TF32 is held to its relFrob gate only.
        np.testing.assert_allclose(got, oracle.mm_torch(x1, x2), rtol=1e-3, atol=1e-2)
    assert oracle.rel_frob(got, oracle.mm_tiled(x1, x2)) <= TOL[variant]


GOLDEN = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "golden.npz"))
GOLDEN_CASES = sorted(k[:-7] for k in GOLDEN.files if k.endswith("_digest"))


@pytest.mark.parametrize("variant", ALL)
@pytest.mark.parametrize("base", GOLDEN_CASES)
def test_golden_vectors(base, variant):
    tag, shape, s = base.split("_")
    m, k, n = map(int, shape.split("x"))
    x1, x2 = (gen.randn_inputs if tag == "randn" else gen.exact_inputs)(m, k, n, int(s[1:]))
    assert gen.digest(x1, x2) == str(GOLDEN[base + "_digest"])
    got = _run(x1, x2, variant)
    if base + "_c" in GOLDEN.files:
        ref = GOLDEN[base + "_c"]
    else:
        got, ref = got[GOLDEN[base + "_rows"]], GOLDEN[base + "_c_rows"]
    if tag == "exact":
        assert np.array_equal(got, ref), f"max diff {np.abs(got - ref).max()}"
    else:
        assert oracle.rel_frob(got, ref) <= TOL[variant]


def _config_inputs(cfg, seed):
    m, k, n, dist = cfg
    g = torch.Generator().manual_seed(seed)
    if dist == "uniform":
        return torch.rand(m, k, generator=g) * 2 - 1, torch.rand(k, n, generator=g) * 2 - 1
    return torch.randn(m, k, generator=g), torch.randn(k, n, generator=g)


@pytest.mark.parametrize("variant", ALL)
@pytest.mark.parametrize("cfg", [gen.CONFIG1, gen.CONFIG2, gen.CONFIG3], ids=["config1", "config2", "config3"])
def test_baseline_configs(cfg, variant):
    m, k, n, _ = cfg
    x1, x2 = _config_inputs(cfg, 11)
    ref = oracle.mm_tiled(x1.numpy(), x2.numpy()) if m * n * k <= 2 ** 31 else oracle.mm_torch(x1, x2)
    got = _run(x1, x2, variant)
    assert np.isfinite(got).all()
    assert oracle.rel_frob(got, ref) <= TOL[variant]


def _sampled_check(x1, x2, got, tol, nrows=8):
    """Sampled rows vs fp64 and the row-checksum identity, both in fp64 on the CPU."""
    m = x1.shape[0]
    rows = torch.unique(torch.linspace(0, m - 1, min(nrows, m)).round().long())
    ref_rows = x1[rows].double() @ x2.double()
    err_rows = oracle.rel_frob(got[rows].numpy(), ref_rows.numpy())
    ref_rs = x1.double() @ x2.double().sum(1)
    err_rs = oracle.rel_frob(got.double().sum(1).numpy(), ref_rs.numpy())
    assert err_rows <= tol, f"sampled rows relFrob {err_rows:.3e}"
    assert err_rs <= max(tol, 1e-5), f"row checksum relFrob {err_rs:.3e}"


@pytest.mark.parametrize("shape", gen.config4_shapes(), ids=lambda s: "x".join(map(str, s)))
def test_config4_sweep(shape):
    m, k, n = shape
    g = torch.Generator().manual_seed(m * 7919 + k * 31 + n)
    x1 = torch.randn(m, k, generator=g)
    x2 = torch.randn(k, n, generator=g)
    d1, d2 = x1.to(DEV), x2.to(DEV)
    variants = ["auto", "simt", "splitk", "3xtf32", "tf32"]
    for v in variants:
        got = ext._matrix_mul(d1, d2, variant=v).cpu()
        _sampled_check(x1, x2, got, TOL[v])


@pytest.mark.parametrize("variant", ("auto", "tf32", "simt"))
def test_operands_past_2_31_elements(variant):
    """int64 indexing: an A and a C of more than 2^31 elements (the reference indexes in
    int32, tilec/jit.py:37).  Rows on both sides of element 2^31 are checked against fp64."""
    tol = TOL[variant]
    g = torch.Generator(device=DEV).manual_seed(31)
    # A: 263,000 x 8192 = 2.15e9 elements (row 262,144 starts at element 2^31).
    a = torch.randn(263000, 8192, device=DEV, generator=g)
    b = torch.randn(8192, 64, device=DEV, generator=g) / 8192 ** 0.5
    c = ext._matrix_mul(a, b, variant=None if variant == "auto" else variant)
    rows = torch.tensor([0, 262143, 262144, 262145, 262999], device=DEV)
    ref = a[rows].double() @ b.double()
    assert ((c[rows].double() - ref).norm() / ref.norm()).item() <= tol
    del a, b, c
    # C: 36,000 x 60,000 = 2.16e9 elements (row 35,792 starts past element 2^31).
    a = torch.randn(36000, 64, device=DEV, generator=g)
    b = torch.randn(64, 60000, device=DEV, generator=g) / 8
    c = ext._matrix_mul(a, b, variant=None if variant == "auto" else variant)
    rows = torch.tensor([0, 35791, 35792, 35999], device=DEV)
    ref = a[rows].double() @ b.double()
    assert ((c[rows].double() - ref).norm() / ref.norm()).item() <= tol
    del a, b, c
    torch.cuda.empty_cache()
    assert _status_clean()


def test_config5_single_gpu():
    m, k, n = 65536, 8192, 8192
    g = torch.Generator(device=DEV).manual_seed(5)
    d1 = torch.randn(m, k, device=DEV, generator=g)
    d2 = torch.randn(k, n, device=DEV, generator=g) / k ** 0.5
    got = ext.matrix_mul(d1, d2)
    rows = torch.unique(torch.linspace(0, m - 1, 16).round().long()).to(DEV)
    ref_rows = (d1[rows].double() @ d2.double()).cpu()
    assert oracle.rel_frob(got[rows].cpu().numpy(), ref_rows.numpy()) <= 1e-5
    ref_rs = (d1.double() @ d2.double().sum(1)).cpu()
    assert oracle.rel_frob(got.double().sum(1).cpu().numpy(), ref_rs.numpy()) <= 1e-5
    assert _status_clean()


@pytest.mark.parametrize("variant", ("splitk", "tf32", "3xtf32"))
@pytest.mark.parametrize("split_k", (1, 2, 3, 7, 16, 64))
def test_forced_split_k(variant, split_k):
    x1, x2 = _config_inputs(gen.CONFIG1, 3)
    got = _run(x1, x2, variant, split_k)
    assert oracle.rel_frob(got, oracle.mm_tiled(x1.numpy(), x2.numpy())) <= TOL[variant]


@pytest.mark.parametrize("variant", ALL)
def test_edge_sizes(variant):
    for (m, k, n) in [(1, 4, 4), (4, 0, 8), (0, 8, 4), (8, 8, 0), (129, 4, 260), (3, 4100, 5 * 4), (300, 8, 1000)]:
        x1, x2 = gen.exact_inputs(m, k, n, 5)
        got = _run(x1, x2, variant)
        assert got.shape == (m, n)
        assert np.array_equal(got, oracle.mm_f64(x1, x2).astype(np.float32))


@pytest.mark.parametrize("variant", ALL)
def test_strided_views_and_guard_band(variant):
    g = torch.Generator().manual_seed(9)
    big1 = torch.randn(300, 520, generator=g).to(DEV)
    big2 = torch.randn(520, 700, generator=g).to(DEV)
    x1 = big1[10:290, 8:520]     # row view: ld = 520, no copy
    x2 = big2[:512, 4:644]       # row view: ld = 700
    if variant in TENSOR:
        assert x1.data_ptr() % 16 == 0 and x2.data_ptr() % 16 == 0
    buf = torch.full((290, 700), float("nan"), device=DEV)
    out = buf[5:285, 30:670]     # guard band around the output, ldc = 700
    ext._matrix_mul(x1, x2, variant=variant, out=out)
    ref = oracle.mm_tiled(x1.cpu().numpy(), x2.cpu().numpy())
    assert oracle.rel_frob(out.cpu().numpy(), ref) <= TOL[variant]
    b = buf.cpu()
    inside = torch.zeros_like(b, dtype=torch.bool)
    inside[5:285, 30:670] = True
    assert torch.isnan(b[~inside]).all(), "a store landed outside [M, N]"
    # transposed operand: copied like tilec/ext.py:59-60
    t = ext._matrix_mul(big2[:512, :300].t(), big2[:512, :644], variant="simt").cpu().numpy()
    assert oracle.rel_frob(t, oracle.mm_tiled(big2[:512, :300].t().contiguous().cpu().numpy(),
                                              big2[:512, :644].cpu().numpy())) <= 1e-5


@pytest.mark.parametrize("variant", ALL)
def test_deterministic(variant):
    x1, x2 = _config_inputs(gen.CONFIG1, 4)
    d1, d2 = x1.to(DEV), x2.to(DEV)
    a = ext._matrix_mul(d1, d2, variant=variant)
    b = ext._matrix_mul(d1, d2, variant=variant)
    assert torch.equal(a, b)


def test_misaligned_rows_are_packed_for_tensor_cores():
    """Rows that are not 16-byte aligned (K, N not multiples of 4, or an odd view offset)
    are packed into an aligned workspace copy so the TMA/tensor-core path still applies."""
    g = torch.Generator(device=DEV).manual_seed(2)
    base = torch.randn(300 * 1001 + 1, device=DEV, generator=g)
    x1 = base[1:].view(300, 1001)[:, :999]        # odd offset and odd row stride
    x2 = torch.randn(999, 333, device=DEV, generator=g)
    ref = oracle.mm_tiled(x1.contiguous().cpu().numpy(), x2.cpu().numpy())
    for v in ("3xtf32", "tf32", "3xtf32_masked", "auto"):
        got = ext._matrix_mul(x1, x2, variant=v).cpu().numpy()
        assert oracle.rel_frob(got, ref) <= TOL[v], v
    assert ext.kernel_plan(torch.empty(1000, 3001, device=DEV), torch.empty(3001, 777, device=DEV))[0] == "3xtf32"


def test_plan_and_status():
    x1 = torch.randn(2048, 2048, device=DEV)
    v, s = ext.kernel_plan(x1, x1)
    assert v in ("simt", "splitk", "tf32", "3xtf32", "3xtf32_masked") and s >= 1
    assert _status_clean()


def test_raw_hi_equals_masked_hi():
    """The tensor core reads only the top 19 bits of a tf32 operand, so feeding the raw fp32
    tile as hi(x) must give exactly the result of feeding the masked copy."""
    for cfg in (gen.CONFIG1, gen.CONFIG2):
        x1, x2 = _config_inputs(cfg, 21)
        d1, d2 = x1.to(DEV), x2.to(DEV)
        a = ext._matrix_mul(d1, d2, variant="3xtf32")
        b = ext._matrix_mul(d1, d2, variant="3xtf32_masked")
        assert torch.equal(a, b)


@pytest.mark.parametrize("k", (1024, 4096, 8192, 16384))
def test_3xtf32_error_flat_in_k(k):
    """Promoted K-chunks keep the 3xTF32 error at fp32 level however long K is."""
    g = torch.Generator(device=DEV).manual_seed(k)
    a = torch.randn(512, k, device=DEV, generator=g)
    b = torch.randn(k, 512, device=DEV, generator=g)
    ref = a.double() @ b.double()
    for v in ("3xtf32", "simt"):
        got = ext._matrix_mul(a, b, variant=v, split_k=1)
        err = ((got.double() - ref).norm() / ref.norm()).item()
        assert err <= 1e-5, f"{v} K={k}: relFrob {err:.3e}"


@pytest.mark.parametrize("chunks", (1, 3, 8))
def test_matrix_mul_host_pipelined(chunks):
    """Host-buffer API: row chunks stream H2D -> GEMM -> D2H on overlapping streams."""
    g = torch.Generator().manual_seed(chunks)
    x1 = torch.randn(1000, 3001, generator=g).pin_memory()
    x2 = torch.randn(3001, 777, generator=g).pin_memory()
    out = ext.matrix_mul_host(x1, x2, chunks=chunks)
    assert out.device.type == "cpu" and out.shape == (1000, 777)
    assert oracle.rel_frob(out.numpy(), oracle.mm_tiled(x1.numpy(), x2.numpy())) <= 1e-5
    with pytest.raises(ValueError, match="host tensors"):
        ext.matrix_mul_host(x1.to(DEV), x2)


@pytest.mark.parametrize("chunks", (4, 16, [100, 156, 3840], [4000, 96], [1536, 2560]))
@pytest.mark.parametrize("shape", [(4096, 1024, 1024), (4096, 2048, 64), (4096, 999, 333)])
def test_matrix_mul_host_equals_device_bitwise(shape, chunks):
    """Chunked host-buffer product (tapered or explicit spans, chunks below one 256-row
    CTA-pair tile included) = the unchunked device product under the same plan, bit for
    bit: every chunk runs the kernel and K split planned for the full product (a stream-K
    plan runs as one pair per tile, since stream-K groups each tile's sums by the tile
    count of the whole product)."""
    m, k, n = shape
    g = torch.Generator().manual_seed(m + k + n)
    x1 = torch.randn(m, k, generator=g).pin_memory()
    x2 = torch.randn(k, n, generator=g).pin_memory()
    d1, d2 = x1.to(DEV), x2.to(DEV)
    v, s = ext.kernel_plan(d1, d2)
    want = ext._matrix_mul(d1, d2, variant=v, split_k=s).cpu()
    assert oracle.rel_frob(want.numpy(), ext.matrix_mul(d1, d2).cpu().numpy()) <= 1e-5
    got = ext.matrix_mul_host(x1, x2, chunks=chunks)
    assert torch.equal(got, want)


@pytest.mark.parametrize("split_k", (1, 2, 3, 7))
@pytest.mark.parametrize("shape", [(1024, 4096, 1024), (300, 2000, 520), (777, 1000, 333)])
def test_cta_pair_kernel(shape, split_k):
    """3xTF32 on 256-row CTA pairs (M >= 256, N > 128): ragged pair tiles, forced K splits,
    raw and masked hi agree bit for bit, error at the fp32 level."""
    m, k, n = shape
    g = torch.Generator(device=DEV).manual_seed(m + k + n + split_k)
    a = torch.randn(m, k, device=DEV, generator=g)
    b = torch.randn(k, n, device=DEV, generator=g)
    got = ext._matrix_mul(a, b, variant="3xtf32", split_k=split_k)
    masked = ext._matrix_mul(a, b, variant="3xtf32_masked", split_k=split_k)
    assert torch.equal(got, masked)
    ref = a.double() @ b.double()
    assert ((got.double() - ref).norm() / ref.norm()).item() <= 1e-5


@pytest.mark.parametrize("shape", [(512, 4096, 64), (100, 8192, 40), (1, 8192, 128), (300, 5000, 200),
                                   (64, 65536, 32), (129, 3000, 96), (7, 20000, 7)])
def test_skinny_split_k(shape):
    """Few output tiles and long K (the library splits K into workspace slabs summed in slice
    order): deterministic, raw and masked hi agree, fp32-level error."""
    m, k, n = shape
    g = torch.Generator(device=DEV).manual_seed(m * 3 + k + n)
    a = torch.randn(m, k, device=DEV, generator=g)
    b = torch.randn(k, n, device=DEV, generator=g)
    got = ext._matrix_mul(a, b, variant="3xtf32")
    again = ext._matrix_mul(a, b, variant="3xtf32")
    masked = ext._matrix_mul(a, b, variant="3xtf32_masked")
    assert torch.equal(got, again) and torch.equal(got, masked)
    ref = a.double() @ b.double()
    assert ((got.double() - ref).norm() / ref.norm()).item() <= 1e-5
    assert _status_clean()


@pytest.mark.parametrize("variant,split_k,stream_k", [("3xtf32", 0, False), ("3xtf32", 29, False),
                                                      ("splitk", 8, False), ("tf32", 5, False),
                                                      ("3xtf32", 1, False), ("simt", 0, False),
                                                      ("3xtf32", 0, True), ("tf32", 0, True)])
def test_back_to_back_launches_in_a_graph(variant, split_k, stream_k):
    """Kernels start while the previous one drains (programmatic dependent launch): a
    CUDA graph of consecutive products that share one workspace and chain through their
    outputs (each next input is the previous output) must equal the same calls run one
    at a time with a device sync between them.  With stream_k the [512 x 64] x [64 x 2048]
    products run in stream-K form, whose ready flags are cleared inside the graph."""
    g = torch.Generator(device=DEV).manual_seed(17)
    m, k, n = 512, 2048, 64
    a = torch.randn(m, k, device=DEV, generator=g)
    bs = [torch.randn(k, n, device=DEV, generator=g) / k ** 0.5 for _ in range(3)]
    w = torch.randn(n, k, device=DEV, generator=g) / n ** 0.5
    outs = [torch.empty(m, n, device=DEV) for _ in range(3)]
    mids = [torch.empty(m, k, device=DEV) for _ in range(3)]

    def chain():
        x = a
        for i in range(3):
            ext._matrix_mul(x, bs[i], variant=variant, split_k=split_k, out=outs[i], stream_k=stream_k)
            ext._matrix_mul(outs[i], w, variant=variant, split_k=split_k, out=mids[i], stream_k=stream_k)
            x = mids[i]

    side = torch.cuda.Stream(device=DEV)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        chain()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain()
    for o in outs + mids:
        o.fill_(float("nan"))
    graph.replay()
    torch.cuda.synchronize()
    got = [o.clone() for o in outs + mids]
    # Reference: the same chain with a full device sync after every call.
    x = a
    for i in range(3):
        ext._matrix_mul(x, bs[i], variant=variant, split_k=split_k, out=outs[i], stream_k=stream_k)
        torch.cuda.synchronize()
        ext._matrix_mul(outs[i], w, variant=variant, split_k=split_k, out=mids[i], stream_k=stream_k)
        torch.cuda.synchronize()
        x = mids[i]
    for g_, r in zip(got, outs + mids):
        assert torch.equal(g_, r)
    del graph
    assert _status_clean()


def test_bounded_wait_times_out_and_context_survives():
    """Failure detection without a fault: a wait on a barrier nothing arrives on gives up
    after its limit (50 ms here), the kernel records TILEC_DEV_STATUS_TIMEOUT and returns;
    the host reads the status, and the same context then computes a product correctly."""
    import time
    lib = _native.load()
    assert _status_clean()
    t0 = time.perf_counter()
    _native.check(lib.tilec_mm_selftest_wait(50_000_000, None), "selftest_wait")
    st = ctypes.c_int32(-1)
    _native.check(lib.tilec_mm_device_status(None, ctypes.byref(st)), "device_status")
    waited = time.perf_counter() - t0
    assert st.value == 1, st.value               # TILEC_DEV_STATUS_TIMEOUT
    assert 0.04 <= waited < 1.5, waited          # gave up near its limit, not the 2 s default
    assert _status_clean()                       # reading cleared it
    x1, x2 = _config_inputs(gen.CONFIG1, 6)
    got = _run(x1, x2, "3xtf32")
    assert oracle.rel_frob(got, oracle.mm_tiled(x1.numpy(), x2.numpy())) <= 1e-5
    assert _status_clean()


def _stored(rows, cols, gen, ld_extra=0):
    """A [rows, cols] row-major device tensor, optionally inside wider rows (ld > cols)."""
    t = torch.randn(rows, cols + ld_extra, device=DEV, generator=gen)
    return t[:, :cols] if ld_extra else t


@pytest.mark.parametrize("variant", ALL)
@pytest.mark.parametrize("ta,tb", [(False, True), (True, False), (True, True)])
@pytest.mark.parametrize("shape,ld_extra", [((512, 4096, 64), 0), ((1000, 3001, 777), 0), ((300, 520, 700), 8),
                                            ((129, 64, 260), 0), ((2048, 1024, 2048), 0), ((7, 33, 5), 3),
                                            ((256, 2048, 40), 4)])
def test_transposed_views_read_in_place(shape, ld_extra, ta, tb, variant):
    """x1 = y.t() and/or x2 = z.t() (column views) go to the library as transposed storage
    (TILEC_MM_TRANS_A / _B): the tensor-core kernels read them in place through MN-major A
    slabs / a K-major B tile, SIMT variants transpose into the workspace.  The product
    equals, bit for bit, the same variant on contiguous copies (what the reference does,
    tilec/ext.py:59-60), and meets the variant's error gate against fp64."""
    m, k, n = shape
    g = torch.Generator(device=DEV).manual_seed(m * 7 + k * 3 + n + 2 * ta + tb)
    x1 = _stored(k, m, g, ld_extra).t() if ta else _stored(m, k, g, ld_extra)
    x2 = _stored(n, k, g, ld_extra).t() if tb else _stored(k, n, g, ld_extra)
    assert (x1.stride(0) == 1) == ta and (x2.stride(0) == 1) == tb
    got = ext._matrix_mul(x1, x2, variant=variant)
    if variant != "auto":
        want = ext._matrix_mul(x1.contiguous(), x2.contiguous(), variant=variant)
        assert torch.equal(got, want)
    ref = x1.double() @ x2.double()
    assert ((got.double() - ref).norm() / ref.norm()).item() <= TOL[variant]
    assert _status_clean()


def test_transposed_views_forced_split_and_pair():
    """Transposed operands through split-K slabs and the CTA-pair kernel (ragged edges)."""
    g = torch.Generator(device=DEV).manual_seed(11)
    y = torch.randn(1500, 777, device=DEV, generator=g)       # x1 = y.t(): [777, 1500]
    z = torch.randn(1000, 1500, device=DEV, generator=g)      # x2 = z.t(): [1500, 1000]
    for split in (1, 3, 7):
        got = ext._matrix_mul(y.t(), z.t(), variant="3xtf32", split_k=split)
        want = ext._matrix_mul(y.t().contiguous(), z.t().contiguous(), variant="3xtf32", split_k=split)
        assert torch.equal(got, want), split
    assert ext.kernel_plan(y.t(), z.t(), variant="3xtf32")[0] == "3xtf32"


NARROW_PAIR_SHAPES = [(1024, 4096, 300), (300, 520, 260), (777, 1000, 384), (513, 3001, 333)]


@pytest.mark.parametrize("shape", NARROW_PAIR_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("variant", ("3xtf32", "tf32"))
def test_pair_tiles_128_columns_wide(shape, variant):
    """CTA pairs on 128-column tiles (M >= 256, 256 < N <= 384): one pair per tile, forced K
    splits and the stream-K form all meet the variant's gate, repeat bit for bit, raw and
    masked hi agree, and a TF32 pair equals the 1-CTA kernel row block by row block (same
    K order per element; the 1-CTA kernel runs 256-column tiles here)."""
    m, k, n = shape
    g = torch.Generator(device=DEV).manual_seed(m + 3 * k + n)
    a = torch.randn(m, k, device=DEV, generator=g)
    b = torch.randn(k, n, device=DEV, generator=g)
    ref = a.double() @ b.double()
    for split, sk in ((1, False), (3, False), (0, True), (0, False)):
        got = ext._matrix_mul(a, b, variant=variant, split_k=split, stream_k=sk)
        again = ext._matrix_mul(a, b, variant=variant, split_k=split, stream_k=sk)
        assert torch.equal(got, again), (split, sk)
        assert ((got.double() - ref).norm() / ref.norm()).item() <= TOL[variant], (split, sk)
        if variant == "3xtf32":
            masked = ext._matrix_mul(a, b, variant="3xtf32_masked", split_k=split, stream_k=sk)
            assert torch.equal(got, masked), (split, sk)
        elif split == 1 and not sk:
            for r0 in range(0, m, 128):
                part = ext._matrix_mul(a[r0:r0 + 128], b, variant="tf32", split_k=1)
                assert torch.equal(got[r0:r0 + 128], part), r0
    if k % 4 == 0 and n % 4 == 0:
        # Column views read in place equal the contiguous operands.
        for split in (1, 3):
            tv = ext._matrix_mul(a.t().contiguous().t(), b.t().contiguous().t(), variant=variant, split_k=split)
            assert torch.equal(tv, ext._matrix_mul(a, b, variant=variant, split_k=split)), split
    assert _status_clean()


def test_pair_tiles_128_columns_wide_batched_and_misaligned():
    """Batched 128-column pair tiles with an odd row stride (both operands packed) equal the
    single products slice by slice."""
    g = torch.Generator(device=DEV).manual_seed(17)
    nb, m, k, n = 3, 600, 1001, 301
    x1 = torch.randn(nb, m, k + 1, device=DEV, generator=g)[:, :, 1:]
    x2 = torch.randn(nb, k, n, device=DEV, generator=g)
    for variant in ("3xtf32", "tf32"):
        for split in (1, 3):
            got = ext.matrix_mul_ex(x1, x2, variant=variant, split_k=split)
            for i in range(nb):
                assert torch.equal(got[i], ext._matrix_mul(x1[i], x2[i], variant=variant, split_k=split)), i
            ref = torch.matmul(x1.double(), x2.double())
            assert ((got.double() - ref).norm() / ref.norm()).item() <= TOL[variant]
    assert _status_clean()


def _ref64(x1, x2, bias=None, act=None):
    r = torch.matmul(x1.double(), x2.double())
    if bias is not None:
        r = r + bias.double()
    if act == "relu":
        r = torch.relu(r)
    elif act == "gelu":
        r = torch.nn.functional.gelu(r)
    return r


@pytest.mark.parametrize("variant", ("simt", "splitk", "tf32", "3xtf32", "3xtf32_masked", "3xmixed"))
@pytest.mark.parametrize("split_k", (1, 3))
@pytest.mark.parametrize("shape", [(5, 300, 520, 700), (3, 512, 2048, 64), (4, 33, 129, 65), (2, 1000, 3001, 777)])
def test_batched_equals_single_products(shape, split_k, variant):
    """matrix_mul_ex on [B, M, K] @ [B, K, N]: every slice equals the single-product call
    with the same variant and K split bit for bit (the batch is a grid dimension, nothing
    else changes), and meets the variant's error gate."""
    nb, m, k, n = shape
    g = torch.Generator(device=DEV).manual_seed(nb * m + k + n + split_k)
    x1 = torch.randn(nb, m, k, device=DEV, generator=g)
    x2 = torch.randn(nb, k, n, device=DEV, generator=g)
    got = ext.matrix_mul_ex(x1, x2, variant=variant, split_k=split_k)
    for b in range(nb):
        one = ext._matrix_mul(x1[b], x2[b], variant=variant, split_k=split_k)
        assert torch.equal(got[b], one), b
    ref = _ref64(x1, x2)
    assert ((got.double() - ref).norm() / ref.norm()).item() <= TOL[variant]
    assert _status_clean()


@pytest.mark.parametrize("variant", ("auto", "simt", "3xtf32", "tf32", "3xmixed"))
def test_batched_shared_transposed_and_misaligned(variant):
    """A shared by the batch (2-D x1), B shared (2-D x2), column views of each slice, and
    batch strides that are not 16-byte multiples (packed for TMA)."""
    g = torch.Generator(device=DEV).manual_seed(5)
    nb, m, k, n = 6, 257, 300, 190
    a2 = torch.randn(m, k, device=DEV, generator=g)
    b3 = torch.randn(nb, k, n, device=DEV, generator=g)
    a3 = torch.randn(nb, m, k, device=DEV, generator=g)
    b2 = torch.randn(k, n, device=DEV, generator=g)
    cases = [(a2, b3), (a3, b2),
             (torch.randn(nb, k, m, device=DEV, generator=g).transpose(1, 2), b3),     # A column views
             (a3, torch.randn(nb, n, k, device=DEV, generator=g).transpose(1, 2)),     # B column views
             (torch.randn(nb, m, k + 1, device=DEV, generator=g)[:, :, 1:], b3)]      # odd offset / stride
    for x1, x2 in cases:
        got = ext.matrix_mul_ex(x1, x2, variant=variant)
        ref = _ref64(x1, x2)
        assert got.shape == ref.shape
        assert ((got.double() - ref).norm() / ref.norm()).item() <= TOL[variant]
    assert _status_clean()


@pytest.mark.parametrize("act", (None, "relu", "gelu"))
@pytest.mark.parametrize("variant,split_k", [("3xtf32", 0), ("3xtf32", 5), ("tf32", 1), ("simt", 0), ("splitk", 4),
                                             ("auto", 0), ("3xmixed", 0), ("3xmixed", 3)])
def test_fused_bias_activation(variant, split_k, act):
    """C = act(A.B + bias) with the epilogue in the GEMM's store (one K slice) or in the
    split-K reduction.  Bias-only and ReLU results are exactly torch's fp32
    act(x1 @ x2 + bias) on the same product; GELU (erf form) within 1e-6 of it."""
    g = torch.Generator(device=DEV).manual_seed(21)
    nb, m, k, n = 3, 384, 1024, 333
    x1 = torch.randn(nb, m, k, device=DEV, generator=g)
    x2 = torch.randn(nb, k, n, device=DEV, generator=g)
    bias = torch.randn(n, device=DEV, generator=g)
    got = ext.matrix_mul_ex(x1, x2, bias=bias, activation=act, variant=variant, split_k=split_k)
    plain = ext.matrix_mul_ex(x1, x2, variant=variant, split_k=split_k)
    want = plain + bias
    if act == "relu":
        want = torch.relu(want)
    if act == "gelu":
        want = torch.nn.functional.gelu(want)
        assert ((got - want).norm() / want.norm()).item() <= 1e-6
    else:
        assert torch.equal(got, want)
    ref = _ref64(x1, x2, bias, act)
    assert ((got.double() - ref).norm() / ref.norm()).item() <= TOL[variant]
    assert _status_clean()


def test_fused_k0_and_large_batch():
    """K = 0 stores act(bias); a batch of 70000 tiny products (more than one launch's grid)
    matches fp64."""
    bias = torch.linspace(-2, 2, 5, device=DEV)
    got = ext.matrix_mul_ex(torch.empty(3, 4, 0, device=DEV), torch.empty(3, 0, 5, device=DEV), bias=bias,
                            activation="relu")
    assert torch.equal(got, torch.relu(bias).expand(3, 4, 5))
    g = torch.Generator(device=DEV).manual_seed(3)
    x1 = torch.randn(70000, 4, 8, device=DEV, generator=g)
    x2 = torch.randn(70000, 8, 4, device=DEV, generator=g)
    for variant in ("simt", "3xtf32"):
        got = ext.matrix_mul_ex(x1, x2, variant=variant)
        ref = _ref64(x1, x2)
        assert ((got.double() - ref).norm() / ref.norm()).item() <= 1e-5, variant
    assert _status_clean()


def test_fused_argument_errors():
    x1 = torch.randn(2, 8, 16, device=DEV)
    x2 = torch.randn(2, 16, 4, device=DEV)
    with pytest.raises(ValueError, match="activation"):
        ext.matrix_mul_ex(x1, x2, activation="tanh")
    with pytest.raises(ValueError, match="bias"):
        ext.matrix_mul_ex(x1, x2, bias=torch.zeros(5, device=DEV))
    with pytest.raises(ValueError, match="batch sizes"):
        ext.matrix_mul_ex(x1, torch.randn(3, 16, 4, device=DEV))
    with pytest.raises(ValueError, match="overlap"):
        ext.matrix_mul_ex(x1, x2, out=torch.empty(8, 4, device=DEV).expand(2, 8, 4))


@pytest.mark.parametrize("shape", [(512, 2048, 512), (1000, 3001, 777), (300, 520, 700)])
@pytest.mark.parametrize("split_k", (1, 3))
def test_tf32_pair_kernel_matches_single_cta(shape, split_k):
    """TF32 on 256-row CTA pairs (M >= 256, N > 128) equals, row block by row block, the
    1-CTA TF32 kernel that a 128-row slice runs on (same K order per element), and keeps
    the TF32 error gate."""
    m, k, n = shape
    g = torch.Generator(device=DEV).manual_seed(m + k + n + 7 * split_k)
    a = torch.randn(m, k, device=DEV, generator=g)
    b = torch.randn(k, n, device=DEV, generator=g)
    got = ext._matrix_mul(a, b, variant="tf32", split_k=split_k)
    for r0 in range(0, m, 128):
        part = ext._matrix_mul(a[r0:r0 + 128], b, variant="tf32", split_k=split_k)
        assert torch.equal(got[r0:r0 + 128], part), r0
    ref = a.double() @ b.double()
    assert ((got.double() - ref).norm() / ref.norm()).item() <= 5e-3
    assert _status_clean()


# ---------------------------------------------------------------- mixed split (tf32 main product, bf16 cross terms)

def _tf32_exact(rows, cols, g):
    """j / 1024 for integer |j| <= 1024: 11 significant bits, exact in tf32 (l(x) = 0)."""
    return (torch.randint(-1024, 1025, (rows, cols), generator=g).float() / 1024).to(DEV)


@pytest.mark.parametrize("shape", [(2048, 2048, 2048), (1000, 3001, 777), (300, 520, 700), (4096, 8192, 512)])
def test_mixed_equals_3xtf32_when_low_parts_vanish(shape):
    """On operands that tf32 holds exactly, l(x) = 0: both cross terms add exact zeros, and
    the tf32 main product runs in the same K order with the same promotion as 3XTF32 (whose
    pair kernel takes 32 of K per stage against the mixed kernel's 16, with the same MMA
    sequence), so with the same K slices the two variants agree bit for bit."""
    m, k, n = shape
    g = torch.Generator().manual_seed(m + k + n)
    a, b = _tf32_exact(m, k, g), _tf32_exact(k, n, g)
    assert ext.kernel_plan(a, b, variant="3xmixed")[0] == "3xmixed"
    split = ext.kernel_plan(a, b, variant="3xtf32")[1]  # same K slices for both (the plans' speed models differ)
    assert torch.equal(ext._matrix_mul(a, b, variant="3xmixed", split_k=split),
                       ext._matrix_mul(a, b, variant="3xtf32", split_k=split))
    assert _status_clean()


@pytest.mark.parametrize("k", (256, 2048, 8192, 16384))
@pytest.mark.parametrize("dist", ("normal", "uniform", "positive"))
def test_mixed_error_gate_and_flat_in_k(k, dist):
    """The bf16 cross terms keep the fp32-class gate (relFrob <= 1e-5 against fp64) on
    zero-mean and on all-positive operands (where rounding errors cannot cancel in sign),
    with K up to 16384; the error stays within 4x of 3XTF32's."""
    g = torch.Generator(device=DEV).manual_seed(k + len(dist))
    if dist == "normal":
        a = torch.randn(512, k, device=DEV, generator=g)
        b = torch.randn(k, 512, device=DEV, generator=g)
    else:
        a = torch.rand(512, k, device=DEV, generator=g)
        b = torch.rand(k, 512, device=DEV, generator=g)
        if dist == "uniform":
            a, b = 2 * a - 1, 2 * b - 1
    ref = a.double() @ b.double()
    mixed = _rel(ext._matrix_mul(a, b, variant="3xmixed"), ref)
    three = _rel(ext._matrix_mul(a, b, variant="3xtf32"), ref)
    assert mixed <= 1e-5, f"3xmixed K={k} {dist}: relFrob {mixed:.3e}"
    assert mixed <= 4 * three + 1e-7, (mixed, three)


def test_mixed_plan_falls_back_where_no_pair_kernel_runs():
    """Shapes outside the CTA-pair kernel (M < 256 or N <= 128) and stream-K requests run
    3XTF32, and the plan says so."""
    a = torch.randn(200, 512, device=DEV)
    b = torch.randn(512, 600, device=DEV)
    assert ext.kernel_plan(a, b, variant="3xmixed")[0] == "3xtf32"
    c = torch.randn(512, 100, device=DEV)
    assert ext.kernel_plan(b.t(), c, variant="3xmixed")[0] == "3xtf32"
    x = torch.randn(2304, 2048, device=DEV)
    info = ext.kernel_plan(x, x.t(), variant="3xmixed", stream_k=True, detail=True)
    assert info["variant"] == "3xmixed" and not info["stream_k"]
    got = ext._matrix_mul(x, x.t(), variant="3xmixed", stream_k=True)
    assert _rel(got, x.double() @ x.t().double()) <= 1e-5


# ---------------------------------------------------------------- stream-K form of the CTA-pair kernel

def _rel(got, ref):
    got, ref = got.double().cpu(), ref.double().cpu()
    return ((got - ref).norm() / ref.norm()).item()


SK_SHAPES = [
    (2048, 2048, 2048),  # 64 tiles, one wave of pairs
    (2304, 2048, 2304),  # 81 tiles: two waves as one pair per tile (AUTO takes stream-K)
    (1000, 3001, 777),   # 16 ragged tiles, about five pairs per tile
    (300, 200, 520),     # 6 tiles of 13 k-blocks: 78 units, one or two per pair
    (257, 64, 300),      # 2 tiles of 4 k-blocks: 8 pairs of one unit
    (4096, 1024, 4608),  # 288 tiles: two whole waves, then stream-K over the rest
]


@pytest.mark.parametrize("variant", SK_VARIANTS)
@pytest.mark.parametrize("shape", SK_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_stream_k_matches_oracle_and_one_pair_per_tile(shape, variant):
    """Stream-K (pairs share out the k-blocks of the tiles and add each tile's partial
    sums in pair order) keeps the variant's error gate against the fp64 product, agrees
    with the one-pair-per-tile form up to fp32 regrouping, and is deterministic."""
    m, k, n = shape
    g = torch.Generator().manual_seed(m + 3 * k + 7 * n)
    x1 = torch.randn(m, k, generator=g)
    x2 = torch.randn(k, n, generator=g)
    a, b = x1.to(DEV), x2.to(DEV)
    info = ext.kernel_plan(a, b, variant=variant, stream_k=True, detail=True)
    assert info["stream_k"] and info["split_k"] == 1, info
    sk = ext._matrix_mul(a, b, variant=variant, stream_k=True)
    dp = ext._matrix_mul(a, b, variant=variant, split_k=1)
    assert _rel(sk, x1.double() @ x2.double()) <= TOL[variant]
    assert _rel(sk, dp) <= 1e-5
    assert torch.equal(sk, ext._matrix_mul(a, b, variant=variant, stream_k=True))
    assert _status_clean()


def test_stream_k_is_auto_choice_where_tiles_leave_pairs_idle():
    """AUTO takes stream-K where one pair per tile would leave most of a wave idle (81
    tiles: two waves on 74 pair slots), not where the last wave is nearly full (2048^3:
    64 tiles in one wave, which stream-K's slower k-blocks would not win back)."""
    x = torch.empty(2304, 2048, device=DEV)
    assert ext.kernel_plan(x, x.t(), detail=True) == {"variant": "3xtf32", "split_k": 1, "stream_k": True,
                                                      "tile_m": None}
    a = torch.empty(2048, 2048, device=DEV)
    assert not ext.kernel_plan(a, a, detail=True)["stream_k"]
    # Whole waves (or K slices asked for) keep one pair per tile.
    big = torch.empty(65536, 8192, device=DEV)
    assert not ext.kernel_plan(big, torch.empty(8192, 8192, device=DEV), detail=True)["stream_k"]
    assert not ext.kernel_plan(a, a, variant="3xtf32", split_k=2, stream_k=True, detail=True)["stream_k"]
    assert not ext.kernel_plan(a, a, variant="3xtf32", split_k=1, detail=True)["stream_k"]
    assert ext.kernel_plan(a, a, variant="3xtf32", split_k=1, stream_k=True, detail=True)["stream_k"]
    # Kernels without a CTA pair ignore the flag.
    assert not ext.kernel_plan(a[:, :64], a[:64, :64], stream_k=True, detail=True)["stream_k"]


@pytest.mark.parametrize("ta,tb", [(False, True), (True, False), (True, True)])
def test_stream_k_transposed_views(ta, tb):
    m, k, n = 1000, 3001, 777
    g = torch.Generator(device=DEV).manual_seed(31 + 2 * ta + tb)
    a = torch.randn(k, m, device=DEV, generator=g).t() if ta else torch.randn(m, k, device=DEV, generator=g)
    b = torch.randn(n, k, device=DEV, generator=g).t() if tb else torch.randn(k, n, device=DEV, generator=g)
    for v in ("3xtf32", "tf32"):
        sk = ext._matrix_mul(a, b, variant=v, stream_k=True)
        assert _rel(sk, ext._matrix_mul(a, b, variant=v, split_k=1)) <= 1e-5
        assert _rel(sk, a.double() @ b.double()) <= TOL[v]
    assert _status_clean()


@pytest.mark.parametrize("act", (None, "relu", "gelu"))
def test_stream_k_batched_fused(act):
    """Stream-K over the tiles of a whole batch (units run across batch boundaries), with
    the bias / activation epilogue applied where each tile is stored, and a shared B."""
    g = torch.Generator(device=DEV).manual_seed(5)
    a = torch.randn(3, 600, 1024, device=DEV, generator=g)
    b = torch.randn(3, 1024, 520, device=DEV, generator=g) / 32
    bias = torch.randn(520, device=DEV, generator=g)
    got = ext.matrix_mul_ex(a, b, bias=bias, activation=act, stream_k=True)
    for i in range(3):
        want = ext.matrix_mul_ex(a[i], b[i], bias=bias, activation=act, split_k=1)
        assert _rel(got[i], want) <= 1e-5, i
        assert _rel(got[i], _ref64(a[i], b[i], bias, act)) <= 1e-5, i
    shared = ext.matrix_mul_ex(a, b[0], bias=bias, activation=act, stream_k=True)
    assert _rel(shared[2], _ref64(a[2], b[0], bias, act)) <= 1e-5
    assert _status_clean()


def test_host_threads_on_separate_streams():
    """The library is stream-ordered and reentrant: four host threads, each on a stream of
    its own, call split-K, CTA-pair, packed (misaligned) and SIMT products at the same
    time; every result equals the same product run alone, bit for bit, and each thread's
    workspace (per stream) keeps its split-K slabs apart from the others'."""
    import threading
    g = torch.Generator(device=DEV).manual_seed(29)
    cases = [((512, 4096, 64), "3xtf32"), ((2048, 1024, 2048), "3xtf32"), ((1000, 3001, 777), "auto"),
             ((300, 700, 500), "splitk")]
    ins = [(torch.randn(m, k, device=DEV, generator=g), torch.randn(k, n, device=DEV, generator=g), v)
           for (m, k, n), v in cases]
    alone = [ext._matrix_mul(a, b, variant=v) for a, b, v in ins]
    torch.cuda.synchronize()
    results = [[] for _ in ins]
    errors = []

    def work(i):
        try:
            a, b, v = ins[i]
            s = torch.cuda.Stream(device=DEV)
            with torch.cuda.stream(s):
                for _ in range(8):
                    results[i].append(ext._matrix_mul(a, b, variant=v))
            s.synchronize()
        except Exception as e:  # noqa: BLE001
            errors.append(repr(e))

    threads = [threading.Thread(target=work, args=(i,)) for i in range(len(ins))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    torch.cuda.synchronize()
    assert not errors, errors
    for r, outs in zip(alone, results):
        assert len(outs) == 8
        for o in outs:
            assert torch.equal(o, r)
    assert _status_clean()


def test_stream_k_concurrent_streams():
    """Two streams run stream-K products at the same time, so the pairs of one launch
    compete for SMs with the other's: a pair waits only on lower-numbered pairs, which the
    block scheduler places first, so every launch completes (no bounded wait runs out) and
    each result equals the same product run alone, bit for bit."""
    g = torch.Generator(device=DEV).manual_seed(23)
    shapes = [(2304, 2048, 2304), (2560, 1024, 2560)]
    ins = [(torch.randn(m, k, device=DEV, generator=g), torch.randn(k, n, device=DEV, generator=g))
           for (m, k, n) in shapes]
    alone = [ext._matrix_mul(a, b, variant="3xtf32", stream_k=True) for a, b in ins]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(device=DEV) for _ in ins]
    outs = [[torch.empty_like(r) for _ in range(4)] for r in alone]
    for s in streams:
        s.wait_stream(torch.cuda.current_stream())
    for rep in range(4):
        for i, ((a, b), s) in enumerate(zip(ins, streams)):
            with torch.cuda.stream(s):
                ext._matrix_mul(a, b, variant="3xtf32", stream_k=True, out=outs[i][rep])
    torch.cuda.synchronize()
    assert _status_clean()
    for r, os_ in zip(alone, outs):
        for o in os_:
            assert torch.equal(o, r)


# ---------------------------------------------------------------- non-finite operands

@pytest.mark.parametrize("variant", ALL)
def test_non_finite_operands(variant):
    """Inf / NaN in x1 or x2 reach exactly the outputs whose dot products contain them, as in
    the reference's fp32 dot (each output is an independent sum): those rows / columns are
    non-finite and every other output is finite and within the variant's gate.  SIMT and
    SPLITK (fp32 FMA) also reproduce the IEEE values, +-Inf or NaN, of `x1 @ x2` on CPU; the
    tensor split variants may give NaN where IEEE gives +-Inf (a zero low part times an
    infinite high part)."""
    g = torch.Generator().manual_seed(31)
    x1 = torch.randn(300, 520, generator=g)
    x2 = torch.randn(520, 700, generator=g)
    x1[5, 17] = float("inf")
    x1[40, 3] = float("nan")
    x1[77, 100] = float("-inf")
    x2[100, 9] = float("-inf")
    x2[200, 650] = float("nan")
    ref = x1 @ x2  # CPU fp32, IEEE
    got = ext._matrix_mul(x1.to(DEV), x2.to(DEV), variant=variant).cpu()
    bad = ~torch.isfinite(ref)
    assert bad.any() and (~bad).any()
    assert torch.equal(~torch.isfinite(got), bad), "non-finite outputs differ from the IEEE pattern"
    if variant in ("simt", "splitk"):
        assert torch.equal(torch.isnan(got), torch.isnan(ref))
        assert torch.equal(got[torch.isinf(ref)], ref[torch.isinf(ref)])
    fin = ~bad
    ref64 = (x1.double() @ x2.double())[fin]
    err = ((got[fin].double() - ref64).norm() / ref64.norm()).item()
    assert err <= TOL[variant], f"{variant}: finite outputs relFrob {err:.3e}"
    assert _status_clean()


@pytest.mark.parametrize("shape,batch,ta,tb", [((2304, 1024, 2304), 0, False, False), ((4096, 512, 4096), 0, False, False),
                                               ((2000, 700, 3000), 0, False, False), ((2304, 1024, 2304), 0, True, True),
                                               ((1024, 256, 2048), 3, False, False)])
def test_tf32_persistent_pairs(shape, batch, ta, tb):
    """TF32 products with more 256 x 256 tiles than pairs fit at once run on the persistent
    pair kernel (two TMEM accumulators per pair, a tile's epilogue overlapping the next
    tile's MMAs).  Its per-tile MMA sequence is the 1-CTA kernel's, so every 128-row block
    equals what the 1-CTA TF32 kernel gives for that slice, bit for bit; and it keeps the
    TF32 gate, with operands read in place when transposed and with batches."""
    m, k, n = shape
    g = torch.Generator(device=DEV).manual_seed(m + n + 3 * batch)
    lead = (batch,) if batch else ()
    a = torch.randn(*lead, m, k, device=DEV, generator=g)
    b = torch.randn(*lead, k, n, device=DEV, generator=g)
    if ta:
        a = a.transpose(-1, -2).contiguous().transpose(-1, -2)
    if tb:
        b = b.transpose(-1, -2).contiguous().transpose(-1, -2)
    if batch:
        got = ext.matrix_mul_ex(a, b, variant="tf32", split_k=1)
    else:
        got = ext._matrix_mul(a, b, variant="tf32", split_k=1)
    for i in range(max(batch, 1)):
        ai, bi, gi = (a[i], b[i], got[i]) if batch else (a, b, got)
        for r0 in range(0, m, 512):
            part = ext._matrix_mul(ai[r0:r0 + 128], bi, variant="tf32", split_k=1)
            assert torch.equal(gi[r0:r0 + 128], part), (i, r0)
    ref = (a.double() @ b.double())
    assert ((got.double() - ref).norm() / ref.norm()).item() <= 5e-3
    assert _status_clean()


@pytest.mark.parametrize("act", (None, "relu", "gelu"))
def test_tf32_persistent_pairs_fused_epilogue(act):
    g = torch.Generator(device=DEV).manual_seed(11)
    a = torch.randn(2304, 512, device=DEV, generator=g)
    b = torch.randn(512, 2304, device=DEV, generator=g)
    bias = torch.randn(2304, device=DEV, generator=g)
    got = ext.matrix_mul_ex(a, b, bias=bias, activation=act, variant="tf32", split_k=1)
    plain = ext._matrix_mul(a, b, variant="tf32", split_k=1) + bias
    want = {None: plain, "relu": torch.relu(plain), "gelu": torch.nn.functional.gelu(plain)}[act]
    assert torch.allclose(got, want, rtol=1e-6, atol=1e-5)
