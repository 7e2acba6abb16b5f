"""tilec_b200.ext -- drop-in for ``tilec.ext`` (tilec/ext.py) on NVIDIA B200.

``matrix_mul(x1, x2)`` keeps the reference's call signature, argument meaning, result
and error behaviour (tilec/ext.py:54-67):

* ``x1`` [M, K] and ``x2`` [K, N] float32 tensors on one CUDA device;
* ``K != K2`` raises ``ValueError("matrix_mul: shapes (..) and (..) don't match")``
  (ext.py:57-58); tensors that are not 2-D fail when their shape is unpacked
  (ext.py:55-56), also with ``ValueError``;
* a non-float32 tensor raises ``TypeError`` (the reference's argument type check,
  tilec/jit.py:34-39);
* the result is a new [M, N] float32 tensor allocated like ``x1.new_empty(M, N)``
  (ext.py:61) holding ``x1 @ x2``.

Where the reference always copies its inputs with ``.contiguous()`` (ext.py:59-60), row
views with unit column stride are passed through with their row stride (no copy);
other layouts are still made contiguous.  There is no CPU path: CPU tensors raise, and
a missing kernel library raises.
"""
import ctypes
import os

import torch

from . import _native
from .language import cdiv  # noqa: F401  (re-exported like tilec/ext.py:3)

# Kernel tile shapes (for callers that size work around them; the library picks per call).
SIMT_TILE = (128, 128, 16)     # BM, BN, BK of the SIMT kernel
TENSOR_TILE = (128, 256, 16)   # BM, BN, BK of the tcgen05 3xTF32 kernel

_ENV_VARIANT = "TILEC_MM_VARIANT"
_ENV_CHECK = "TILEC_MM_CHECK"


# Per-call host cost matters for small products, so the hot path reads the environment
# through the bytes-keyed dict behind os.environ on POSIX (os.environ.get re-encodes the
# key and decodes the value on every call: ~0.5 us against ~0.05 us) and takes the current
# stream as a raw handle (torch.cuda.current_stream() builds a Stream object: ~2 us).
_ENV_DATA = getattr(os.environ, "_data", None) if os.name == "posix" else None
_ENV_VARIANT_B = _ENV_VARIANT.encode()
_ENV_CHECK_B = _ENV_CHECK.encode()
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _default_variant():
    if _ENV_DATA is not None:
        v = _ENV_DATA.get(_ENV_VARIANT_B)
        return "auto" if v is None else v.decode()
    return os.environ.get(_ENV_VARIANT, "auto")


def _check_enabled():
    """TILEC_MM_CHECK=1: every call synchronises its stream and raises on a device fault."""
    if _ENV_DATA is not None:
        v = _ENV_DATA.get(_ENV_CHECK_B)
        return v is not None and v not in (b"", b"0")
    return os.environ.get(_ENV_CHECK, "0") not in ("", "0")


def _current_stream(index):
    """Raw handle of the current stream of CUDA device `index`."""
    if _raw_stream is not None:
        return _raw_stream(index)
    return torch.cuda.current_stream(index).cuda_stream


def _check_operand(x):
    if x.dtype != torch.float32:
        raise TypeError(f"unsupported kernel argument of dtype {x.dtype} (use float32 tensors and ints)")


def _operand(x):
    """(tensor, leading stride, transposed) for a 2-D operand, copying only when it must.

    A row view (unit column stride) passes as is.  A column view (unit row stride, e.g.
    y.t() of a row-major y) passes as the transposed storage it is: the tensor-core
    kernels read it in place (TILEC_MM_TRANS_A / _B).  The reference makes both
    contiguous (tilec/ext.py:59-60); anything else is still copied here."""
    r, c = x.shape
    s0, s1 = x.stride()
    if (c <= 1 or s1 == 1) and (r <= 1 or s0 >= max(c, 1)):
        return x, (s0 if r > 1 else max(c, 1)), False
    if s0 == 1 and s1 >= r:
        return x, s1, True
    x = x.contiguous()
    return x, max(c, 1), False


def _check_out(out, M, N, device):
    """`device`: a torch.device or a CUDA device index."""
    if out.dtype != torch.float32:
        raise TypeError(f"matrix_mul: out must be float32, got {out.dtype}")
    index = device if isinstance(device, int) else device.index
    if not out.is_cuda or out.get_device() != index:
        raise ValueError(f"matrix_mul: out is on {out.device}, inputs on cuda:{index}")
    if out.shape != (M, N):
        raise ValueError(f"matrix_mul: out has shape {tuple(out.shape)}, expected {(M, N)}")
    s0, s1 = out.stride()
    if not ((N <= 1 or s1 == 1) and (M <= 1 or s0 >= max(N, 1))):
        raise ValueError("matrix_mul: out must have unit column stride and non-overlapping rows")
    return s0 if M > 1 else max(N, 1)


_WS_BYTES = {}   # (shape, strides, 16-byte alignment of A/B/C, variant, split) -> workspace bytes
_WS_BYTES_MAX = 4096
_WS = {}         # (device index, stream handle) -> grow-only workspace tensor
_installed = False
_fast = None     # _native.fast(), fetched on the first launch


def _workspace(dev, stream, nbytes):
    """A workspace of >= nbytes for work ordered on `stream` (reused across calls)."""
    key = (dev.index, stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() * 4 < nbytes:
        ws = torch.empty((nbytes + 4095) // 4096 * 1024, dtype=torch.float32, device=dev)
        _WS[key] = ws
    return ws


def _launch(a, lda, b, ldb, out, ldc, M, N, K, variant, split_k, flags=0):
    global _installed, _fast
    lib = _native.load()
    if not _installed:
        from . import select  # installs the B200 selection table on first use
        select.ensure_installed()
        _fast = _native.fast()
        _installed = True
    cfg = _native.make_cfg(variant, split_k, flags)
    pa, pb, pc = a.data_ptr(), b.data_ptr(), out.data_ptr()
    index = out.get_device()
    prev = torch.cuda.current_device()
    switch = prev != index
    if switch:
        torch.cuda.set_device(index)
    try:
        stream = _current_stream(index)
        key = (M, N, K, lda, ldb, ldc, (pa | pb << 4 | pc << 8) & 0xF0F0F, cfg.variant, cfg.split_k, flags, index)
        ws_bytes = _WS_BYTES.get(key)
        if ws_bytes is None:
            ws_bytes = lib.tilec_mm_workspace_bytes(pa, pb, pc, M, N, K, lda, ldb, ldc, ctypes.byref(cfg))
            if len(_WS_BYTES) >= _WS_BYTES_MAX:  # a process that sees many shapes: start over
                _WS_BYTES.clear()
            _WS_BYTES[key] = ws_bytes
        ws_ptr = _workspace(out.device, stream, ws_bytes).data_ptr() if ws_bytes else None
        if _fast is not None:  # the same C ABI call without ctypes' argument conversion
            rc = _fast.mm(pa, pb, pc, M, N, K, lda, ldb, ldc, cfg.variant, cfg.split_k, cfg.flags, ws_ptr, ws_bytes,
                          stream)
        else:
            rc = lib.tilec_mm_f32(pa, pb, pc, M, N, K, lda, ldb, ldc, ctypes.byref(cfg), ws_ptr, ws_bytes, stream)
        _native.check(rc, "tilec_mm_f32")
        if _check_enabled():
            check_device(stream)
    finally:
        if switch:
            torch.cuda.set_device(prev)
    return out


def _tile_flags(tile_m):
    if tile_m is None:
        return 0
    if tile_m == 64:
        return _native.TILE_M64
    if tile_m == 128:
        return _native.TILE_M128
    raise ValueError(f"tile_m must be None, 64 or 128, got {tile_m!r}")


def _matrix_mul(x1, x2, variant=None, split_k=0, out=None, stream_k=False, tile_m=None):
    """matrix_mul with explicit kernel choice.

    variant: None (= $TILEC_MM_VARIANT or "auto"), "simt", "splitk", "tf32", "3xtf32",
    "3xtf32_masked", "3xmixed" (3xtf32 with its two cross terms on the bf16 tensor pipe;
    CTA-pair shapes only, others run "3xtf32").  split_k: K slices for split variants
    (0 = library choice; 1 = none, which also rules out stream-K).  stream_k: run the
    CTA-pair kernel in its stream-K form
    whenever it is the kernel and split_k <= 1 (the library picks it by itself where it
    pays).  tile_m: None (library choice), 64 or 128 rows per tile of the 1-CTA tensor-core
    kernel (64 also rules out the CTA pair).  out: optional preallocated [M, N] float32
    result (unit column stride).
    """
    M, K = x1.shape
    K2, N = x2.shape
    if K != K2:
        raise ValueError(f"matrix_mul: shapes {tuple(x1.shape)} and {tuple(x2.shape)} don't match")
    _check_operand(x1)
    _check_operand(x2)
    if not (x1.is_cuda and x2.is_cuda):
        raise ValueError(f"matrix_mul: inputs must be CUDA tensors (got {x1.device} and {x2.device}); "
                         "tilec_b200 has no CPU path")
    index = x1.get_device()
    if x2.get_device() != index:
        raise ValueError(f"matrix_mul: inputs on different devices ({x1.device}, {x2.device})")
    a, lda, ta = _operand(x1)
    b, ldb, tb = _operand(x2)
    if out is None:
        out = x1.new_empty(M, N)
        ldc = max(N, 1)
    else:
        ldc = _check_out(out, M, N, index)
    if M == 0 or N == 0:
        return out
    flags = ((_native.TRANS_A if ta else 0) | (_native.TRANS_B if tb else 0) | (_native.STREAM_K if stream_k else 0)
             | (_tile_flags(tile_m) if tile_m is not None else 0))
    return _launch(a, lda, b, ldb, out, ldc, M, N, K, variant or _default_variant(), split_k, flags)


def matrix_mul(x1, x2):
    """C = x1 @ x2 for float32 CUDA tensors x1 [M, K], x2 [K, N] (tilec/ext.py:66-67).

    Kernels never trap: a device-side wait that gives up (see tilec_mm.h) leaves NaN in
    the output tiles it did not finish and sets the device status word.  Set
    TILEC_MM_CHECK=1 (or call check_device()) to have it raised as a TilecError."""
    return _matrix_mul(x1, x2)


def _matrix_mul_tiled(x1, x2, BM=64, BN=64, BK=16):
    """The reference's tiled entry point (tilec/ext.py:54-63) with its signature.  BM, BN
    and BK name the reference kernel's tile (64 x 64 x 16); the B200 kernels choose their
    own tiles per shape, so the values are checked and otherwise unused."""
    for name, v in (("BM", BM), ("BN", BN), ("BK", BK)):
        if not isinstance(v, int) or v <= 0:
            raise ValueError(f"_matrix_mul_tiled: {name} must be a positive int, got {v!r}")
    return _matrix_mul(x1, x2)


# ---------------------------------------------------------------- reference host helpers
# The reference's module-level sizing helpers keep their names, signatures and results
# (tilec/ext.py:10, 29-51), so code written against tilec.ext keeps working.  They describe
# the reference's own Metal kernel configurations (row split, row join, block size); the
# B200 kernels' launch configurations are kernel_plan() and kernel_configs() below.
MAX_BLOCK = 4096
SPLITS = (1, 2, 4, 8, 16, 32, 64)
JOINS = (1, 2, 4, 8)
BLOCKS = (256, 1024, 4096)


def plan(N, block=None):
    """(block, chunks) for a row of N elements (tilec/ext.py:29-34): unless given, block is
    the smallest power of 4 that reaches min(N, MAX_BLOCK), and chunks = cdiv(N, block)."""
    if block is None:
        block = 1
        while block < min(N, MAX_BLOCK):
            block *= 4
    return block, cdiv(N, block)


def _candidate_blocks(n):
    """Block sizes tried for rows of n elements (tilec/ext.py:43-45): the listed sizes below
    plan(n)'s block that leave at most 16 chunks, then plan(n)'s block itself."""
    top = plan(n)[0]
    return [b for b in BLOCKS if b < top and cdiv(n, b) <= 16] + [top]


def mm_configs(M1, N, M2):
    """(split, join, block) triples of the reference's tuner (tilec/ext.py:48-51): a split
    p > 1 needs N // p >= 32, a join r > 1 needs M1 >= r, and blocks come from
    _candidate_blocks(cdiv(N, p)).  M2 does not restrict the space (as in the reference)."""
    out = []
    for p in SPLITS:
        if p > 1 and N // p < 32:
            continue
        for r in JOINS:
            if r > 1 and M1 < r:
                continue
            out.extend((p, r, b) for b in _candidate_blocks(cdiv(N, p)))
    return out


def check_device(stream=None):
    """Read and clear the device status word of the current device (synchronising the
    current stream, or `stream`); raise TilecError(TILEC_ERR_DEVICE) if a kernel recorded a
    fault there (a bounded wait that gave up, a bad launch shape, an unexpected TMEM
    address).  Returns the (zero) status word otherwise."""
    lib = _native.load()
    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    st = ctypes.c_int32(0)
    _native.check(lib.tilec_mm_device_status(s, ctypes.byref(st)), "tilec_mm_device_status")
    if st.value:
        raise _native.TilecError(_native.TILEC_ERR_DEVICE, f"device status word {st.value:#x} "
                                 f"({_native.status_bits(st.value)})")
    return 0


def _batched_operand(x):
    """(tensor, leading stride, transposed, batch stride, batch count or None) for a 2-D
    operand or a 3-D batch of them whose slices are all row views or all column views
    (copied to contiguous otherwise)."""
    if x.dim() == 2:
        t, ld, trans = _operand(x)
        return t, ld, trans, 0, None
    if x.dim() != 3:
        raise ValueError(f"matrix_mul_ex: operands must be 2-D or 3-D, got shape {tuple(x.shape)}")
    nb, r, c = x.shape
    sb, sr, sc = x.stride()
    if (c <= 1 or sc == 1) and (r <= 1 or sr >= max(c, 1)):
        return x, (sr if r > 1 else max(c, 1)), False, sb, nb
    if sr == 1 and sc >= r:
        return x, sc, True, sb, nb
    x = x.contiguous()
    return x, max(c, 1), False, r * c, nb


def matrix_mul_ex(x1, x2, bias=None, activation=None, out=None, variant=None, split_k=0, stream_k=False,
                  tile_m=None):
    """act(x1 @ x2 + bias), batched: the fused, batched form of matrix_mul.

    x1 [M, K] or [B, M, K]; x2 [K, N] or [B, K, N] (a 2-D operand is shared by every
    product of the batch); bias: None or a float32 [N] tensor added per column;
    activation: None, "relu" or "gelu" (exact erf form).  Returns (or writes into `out`)
    [M, N] or [B, M, N].  One library call (tilec_mm_f32_ex): the batch is a grid dimension
    of the kernels and the epilogue runs where C is stored.  Row views and column views
    (.t() / .transpose(-1, -2)) of each slice are read in place, as in matrix_mul.
    variant / split_k / stream_k / tile_m as in _matrix_mul (stream-K shares out the tiles
    of the whole batch).
    """
    _check_operand(x1)
    _check_operand(x2)
    if x1.device.type != "cuda" or x2.device.type != "cuda" or x1.device != x2.device:
        raise ValueError(f"matrix_mul_ex: inputs must be CUDA tensors on one device (got {x1.device} and {x2.device})")
    M, K = x1.shape[-2:]
    K2, N = x2.shape[-2:]
    if K != K2:
        raise ValueError(f"matrix_mul: shapes {tuple(x1.shape)} and {tuple(x2.shape)} don't match")
    a, lda, ta, sa, na = _batched_operand(x1)
    b, ldb, tb, sb, nbb = _batched_operand(x2)
    if na is not None and nbb is not None and na != nbb:
        raise ValueError(f"matrix_mul_ex: batch sizes {na} and {nbb} don't match")
    nb = na if na is not None else nbb
    if activation not in _native.ACTIVATIONS:
        raise ValueError(f"matrix_mul_ex: unknown activation {activation!r}; expected None, 'relu' or 'gelu'")
    if bias is not None:
        if bias.dtype != torch.float32 or bias.dim() != 1 or bias.shape[0] != N or bias.device != x1.device:
            raise ValueError(f"matrix_mul_ex: bias must be a float32 [{N}] tensor on {x1.device}")
        bias = bias.contiguous()
    shape = (M, N) if nb is None else (nb, M, N)
    if out is None:
        out = x1.new_empty(shape)
    elif tuple(out.shape) != shape or out.dtype != torch.float32 or out.device != x1.device:
        raise ValueError(f"matrix_mul_ex: out must be a float32 {shape} tensor on {x1.device}")
    c2 = out if nb is None else out[0]
    ldc = _check_out(c2, M, N, x1.device) if M * N else max(N, 1)
    sc = 0 if nb is None else out.stride(0)
    if M == 0 or N == 0 or nb == 0:
        return out
    nbatch = 1 if nb is None else nb
    if nbatch > 1 and sc < (M - 1) * ldc + N:
        raise ValueError("matrix_mul_ex: the batches of out overlap")
    flags = ((_native.TRANS_A if ta else 0) | (_native.TRANS_B if tb else 0) | (_native.STREAM_K if stream_k else 0)
             | _tile_flags(tile_m))
    lib = _native.load()
    from . import select
    select.ensure_installed()
    cfg = _native.make_cfg(variant or _default_variant(), split_k, flags, _native.ACTIVATIONS[activation])
    pa, pb, pc = a.data_ptr(), b.data_ptr(), out.data_ptr()
    dev = out.device
    with torch.cuda.device(dev):
        stream = _current_stream(dev.index)
        ws_bytes = lib.tilec_mm_workspace_bytes_ex(pa, pb, pc, M, N, K, lda, ldb, ldc, nbatch, sa, sb, sc,
                                                   ctypes.byref(cfg))
        ws_ptr = _workspace(dev, stream, ws_bytes).data_ptr() if ws_bytes else None
        rc = lib.tilec_mm_f32_ex(pa, pb, pc, bias.data_ptr() if bias is not None else None, M, N, K, lda, ldb, ldc,
                                 nbatch, sa, sb, sc, ctypes.byref(cfg), ws_ptr, ws_bytes, stream)
        _native.check(rc, "tilec_mm_f32_ex")
        if _check_enabled():
            check_device(stream)
    return out


def kernel_plan(x1, x2, variant=None, split_k=0, stream_k=False, detail=False, tile_m=None):
    """The (variant name, split_k) that matrix_mul would launch for these operands; with
    detail=True a dict that also says whether the pair kernel runs in its stream-K form and
    the rows per tile of the 1-CTA tensor-core kernel (None for other kernels)."""
    M, K = x1.shape
    _, N = x2.shape
    a, lda, ta = _operand(x1)
    b, ldb, tb = _operand(x2)
    lib = _native.load()
    from . import select
    select.ensure_installed()
    flags = ((_native.TRANS_A if ta else 0) | (_native.TRANS_B if tb else 0) | (_native.STREAM_K if stream_k else 0)
             | _tile_flags(tile_m))
    cfg = _native.make_cfg(variant or _default_variant(), split_k, flags)
    res = _native.MMConfig()
    with torch.cuda.device(x1.device):
        rc = lib.tilec_mm_plan(a.data_ptr(), b.data_ptr(), None, M, N, K, lda, ldb, max(N, 1),
                               ctypes.byref(cfg), ctypes.byref(res))
    _native.check(rc, "tilec_mm_plan")
    name = _native.VARIANT_NAMES.get(res.variant, res.variant)
    if detail:
        tm = 64 if res.flags & _native.TILE_M64 else (128 if res.flags & _native.TILE_M128 else None)
        return {"variant": name, "split_k": res.split_k, "stream_k": bool(res.flags & _native.STREAM_K),
                "tile_m": tm}
    return name, res.split_k


def kernel_configs(M, K, N):
    """Candidate (variant, split_k) launch configs for an [M,K]x[K,N] product.

    B200 counterpart of the reference's config space (tilec/ext.py:48-51), which the
    tuner sweeps (tilec/tune.py:82).  Tensor-core variants pack operands whose rows are
    not 16-byte aligned into an aligned workspace copy first.
    """
    out = [("simt", 1)]
    tiles = cdiv(M, 128) * cdiv(N, 128 if N > 64 else 64)
    for s in (2, 4, 8, 16, 32, 64):
        if K >= s * 128 and tiles * s <= 4 * 148:
            out.append(("splitk", s))
    tiles_tc = cdiv(M, 128) * cdiv(N, 256 if N > 128 else (128 if N > 64 else 64))
    for v in ("3xtf32", "tf32"):
        out.append((v, 1))
        for s in (2, 4, 8, 16, 32, 64):
            if K >= s * 128 and tiles_tc * s <= 2 * 148:
                out.append((v, s))
    return out


_SIDE_STREAMS = {}


def _side_streams(dev):
    """(h2d, d2h) copy streams of a device, created once."""
    if dev not in _SIDE_STREAMS:
        _SIDE_STREAMS[dev] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return _SIDE_STREAMS[dev]


def _row_chunks(M, chunks, align=256, taper=True, min_rows=1024):
    """Row spans for pipelined_rows.  `chunks` is a count (equal spans rounded up to
    `align` rows, one 256-row CTA-pair tile, and at least `min_rows` rows so each span's
    GEMM still fills the GPU) or an explicit sequence of row counts.

    With taper, the first and last equal spans are cut into quarters, a quarter and a half
    (head: 1/4, 1/4, 1/2; tail: 1/2, 1/4, 1/4).  While host<->device copies bound the
    pipeline, a step ends at "last H2D + GEMM of the last span + its D2H" and the first
    GEMM waits for the first span, so short end spans shorten the fill and the drain while
    the middle spans stay large enough to fill whole waves of the GPU."""
    if not isinstance(chunks, int):
        sizes = [int(c) for c in chunks]
        if any(c <= 0 for c in sizes) or sum(sizes) != M:
            raise ValueError(f"chunk sizes {sizes} must be positive and sum to {M}")
    else:
        n = max(1, min(int(chunks), max(1, M // max(align, min_rows))))
        step = -(-M // n)
        step = -(-step // align) * align
        sizes = [min(step, M - r) for r in range(0, M, step)]
        if taper and len(sizes) >= 3:
            q = (step // 4) // align * align
            if q >= align:
                head = [q, q, sizes[0] - 2 * q]
                last = sizes[-1]
                half, quarter = (last // 2) // align * align, (last // 4) // align * align
                tail = [half, quarter, last - half - quarter] if quarter >= align else [last]
                sizes = head + sizes[1:-1] + tail
    spans, r = [], 0
    for c in sizes:
        spans.append((r, r + c))
        r += c
    return spans


def pipelined_rows(h_x1, h_out, dev, make_compute, chunks=16, before=None, sync=True, h2d_hook=None):
    """Stream host rows through the GPU: H2D of chunk i+1, compute(chunk i) and D2H of
    chunk i-1 overlap on three streams (copies on two side streams, compute on the current
    stream).  make_compute(d_x1, d_out) receives the full-size device buffers (so the
    caller can plan the unchunked product) and returns compute(d_x1_rows, d_out_rows),
    which launches the work for one chunk of rows; before() (optional) runs on the
    current stream first (e.g. staging x2).  h2d_hook(i) (optional) runs on the H2D stream
    right before chunk i's copy, and h2d_hook(None) after the last one (e.g. copies of x2
    interleaved with x1's rows).  `chunks`: see _row_chunks."""
    M, K = h_x1.shape
    N = h_out.shape[1]
    cur = torch.cuda.current_stream(dev)
    h2d, d2h = _side_streams(dev)
    d_x1 = torch.empty(M, K, dtype=torch.float32, device=dev)
    d_out = torch.empty(M, N, dtype=torch.float32, device=dev)
    compute = make_compute(d_x1, d_out)
    h2d.wait_stream(cur)
    d2h.wait_stream(cur)
    spans = _row_chunks(M, chunks)
    ev_in = []
    with torch.cuda.stream(h2d):
        for i, (r0, r1) in enumerate(spans):
            if h2d_hook is not None:
                h2d_hook(i)
            d_x1[r0:r1].copy_(h_x1[r0:r1], non_blocking=True)
            ev_in.append(h2d.record_event())
        if h2d_hook is not None:
            h2d_hook(None)
    if before is not None:
        before()
    for (r0, r1), e in zip(spans, ev_in):
        cur.wait_event(e)
        compute(d_x1[r0:r1], d_out[r0:r1])
        d2h.wait_event(cur.record_event())
        with torch.cuda.stream(d2h):
            h_out[r0:r1].copy_(d_out[r0:r1], non_blocking=True)
    d_x1.record_stream(h2d)
    d_out.record_stream(d2h)
    cur.wait_stream(d2h)
    if sync:
        cur.synchronize()
    return h_out


def matrix_mul_host(x1, x2, out=None, chunks=16, device=None, sync=True):
    """C = x1 @ x2 for float32 tensors in host memory, computed on the GPU.

    The same product as matrix_mul, for data that lives on the host: x2 is copied once,
    then row chunks of x1 are copied in, multiplied and copied back with the three
    overlapping (use pinned tensors for asynchronous copies).  `chunks` is a count
    (tapered spans, see _row_chunks) or a sequence of row counts.  Returns `out` (a new pinned
    [M, N] tensor by default), complete when the call returns (sync=True) or once the
    current stream is synchronised (sync=False).
    """
    M, K = x1.shape
    K2, N = x2.shape
    if K != K2:
        raise ValueError(f"matrix_mul: shapes {tuple(x1.shape)} and {tuple(x2.shape)} don't match")
    _check_operand(x1)
    _check_operand(x2)
    if x1.device.type != "cpu" or x2.device.type != "cpu":
        raise ValueError("matrix_mul_host: x1 and x2 must be host tensors (use matrix_mul for CUDA tensors)")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32, pin_memory=True)
    if M == 0 or N == 0:
        return out
    x1 = x1.contiguous()
    with torch.cuda.device(dev):
        d_x2 = torch.empty(K, N, dtype=torch.float32, device=dev)
        d_x2.copy_(x2.contiguous(), non_blocking=True)
        pipelined_rows(x1, out, dev, lambda d_x1, d_out: chunk_compute(d_x1, d_x2), chunks=chunks, sync=sync)
    return out


def chunk_compute(d_x1, d_x2, variant=None, split_k=0):
    """compute(rows_of_x1, rows_of_out) for one row chunk of the product d_x1 @ d_x2 with
    the kernel and K split that the unchunked product uses (planned once on the full-size
    buffers), so a chunked product equals the unchunked one bit for bit."""
    info = kernel_plan(d_x1, d_x2, variant=variant, split_k=split_k, detail=True)
    v, s, tm = info["variant"], info["split_k"], info["tile_m"]
    return lambda a, c: _matrix_mul(a, d_x2, variant=v, split_k=s, out=c, tile_m=tm)
