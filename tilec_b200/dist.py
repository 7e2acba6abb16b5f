"""Row-sharded matrix_mul across the GPUs of one box (one process per GPU).

The reference has no multi-GPU path.  For large M, C = x1 @ x2 splits into independent
row blocks C[r] = x1[r] @ x2 once every GPU holds x2, so the only exchange is
replicating x2 from one rank:

* rank r owns rows ``shard_rows(M, world, r)`` of x1 and of C;
* x2 ([K, N], on rank ``src``) is cut into ``panels`` column panels; rank ``src`` packs
  panel p into a contiguous [K, w_p] buffer and NCCL broadcasts it into every rank's
  own buffer (kernels only ever read local memory);
* rank ``src`` packs and broadcasts panel by panel, so the broadcast of panel p waits
  only for its own pack and the pack of panel p+1 overlaps it; the GEMM of panel p waits
  for broadcast p only (``Work.wait()`` orders the compute stream behind the NCCL
  stream; no host blocking and no device spin-wait), so broadcast p+1 overlaps GEMM p;
* panel p's GEMM writes C[:, n0:n1] in place (ldc = N): no reduction, no extra traffic;
* the output stays sharded, or is all-gathered on request (``gather=True``).

Process groups use the backend of the caller (NCCL on GPUs; the partition, broadcast
and gather logic is also exercised with gloo on CPU ranks in the tests).
"""
import ctypes

import torch
import torch.distributed as dist

_CUDART = None


def _cudart():
    """The CUDA runtime torch loaded (same soname, so the same runtime state and streams)."""
    global _CUDART
    if _CUDART is None:
        torch.cuda.init()
        lib = ctypes.CDLL("libcudart.so.12")
        lib.cudaMemcpy2DAsync.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
                                          ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
        lib.cudaMemcpy2DAsync.restype = ctypes.c_int
        _CUDART = lib
    return _CUDART


def copy_columns_h2d(dst, h_src, n0, n1, stream=None):
    """dst (a contiguous [K, n1 - n0] device tensor) <- h_src[:, n0:n1] (a host [K, N] tensor
    with unit column stride), as one 2-D copy on `stream` (default: the current stream):
    K rows of (n1 - n0) * 4 bytes, source pitch h_src.stride(0) * 4.  Asynchronous when
    h_src is pinned; a column panel of a row-major x2 then needs no host-side packing."""
    K = h_src.shape[0]
    w = n1 - n0
    if tuple(dst.shape) != (K, w) or not dst.is_contiguous() or dst.dtype != h_src.dtype:
        raise ValueError(f"copy_columns_h2d: dst must be a contiguous [{K}, {w}] tensor of {h_src.dtype}")
    if K == 0 or w == 0:
        return dst
    if h_src.stride(1) != 1 and w > 1:
        dst.copy_(h_src[:, n0:n1], non_blocking=False)
        return dst
    s = stream if stream is not None else torch.cuda.current_stream(dst.device)
    es = h_src.element_size()
    rc = _cudart().cudaMemcpy2DAsync(dst.data_ptr(), w * es, h_src.data_ptr() + n0 * es, h_src.stride(0) * es,
                                     w * es, K, 1, s.cuda_stream)  # 1 = cudaMemcpyHostToDevice
    if rc != 0:
        raise RuntimeError(f"copy_columns_h2d: cudaMemcpy2DAsync failed with error {rc}")
    return dst


def shard_rows(M, world, rank):
    """[start, stop) of the rows rank owns: near-equal blocks, the first M % world ranks get one extra."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(M, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def panel_bounds(N, panels, align=256, taper=False):
    """Split [0, N) into <= panels contiguous column ranges, widths multiples of `align`
    except the last (tile-aligned panels keep the GEMM's N tiles whole).

    taper: widths grow twofold from panel to panel (shares 1, 2, 4, ... of N), so the first
    panel, whose broadcast no GEMM can hide, is short, and each later broadcast runs under
    the GEMM of a panel half its width."""
    if N <= 0:
        return []
    panels = max(1, int(panels))
    if taper and panels > 1:
        total = (1 << panels) - 1
        out, n0 = [], 0
        for i in range(panels):
            n1 = N if i == panels - 1 else min(N, -(-(N * ((1 << (i + 1)) - 1) // total) // align) * align)
            if n1 > n0:
                out.append((n0, n1))
                n0 = n1
        return out
    width = -(-N // panels)
    width = -(-width // align) * align
    out = []
    n0 = 0
    while n0 < N:
        n1 = min(N, n0 + width)
        out.append((n0, n1))
        n0 = n1
    return out


def pack_panels(x2, bounds, bufs):
    """Copy column panels of x2 into contiguous per-panel buffers (source rank only)."""
    for (n0, n1), b in zip(bounds, bufs):
        b.copy_(x2[:, n0:n1])


def broadcast_panels(bufs, src=0, group=None):
    """Enqueue one async broadcast per panel; returns the Work handles in panel order."""
    return [dist.broadcast(b, src=src, group=group, async_op=True) for b in bufs]


def gather_rows(c_shard, M, group=None):
    """All-gather row shards (possibly of unequal length) into the full [M, N] result."""
    world = dist.get_world_size(group)
    sizes = [shard_rows(M, world, r) for r in range(world)]
    longest = max(b - a for a, b in sizes)
    N = c_shard.shape[1]
    padded = c_shard
    if c_shard.shape[0] != longest:
        padded = c_shard.new_zeros(longest, N)
        padded[: c_shard.shape[0]].copy_(c_shard)
    full = c_shard.new_empty(world * longest, N)
    dist.all_gather_into_tensor(full, padded.contiguous(), group=group)
    parts = [full[r * longest: r * longest + (b - a)] for r, (a, b) in enumerate(sizes)]
    return torch.cat(parts, 0)


class RowShardedMatmul:
    """C[rows of this rank] = x1_shard @ x2, with x2 broadcast from ``src`` in panels.

    Buffers for x2's panels are allocated once and reused across calls.
    """

    def __init__(self, K, N, panels=2, group=None, src=0, device=None, taper=False):
        self.K, self.N = int(K), int(N)
        self.group = group
        self.src = src
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.bounds = panel_bounds(self.N, panels if self.world > 1 else 1, taper=taper)
        self.bufs = [torch.empty(self.K, n1 - n0, dtype=torch.float32, device=self.device)
                     for (n0, n1) in self.bounds] if self.world > 1 else []
        self.gemm_launches_per_call = len(self.bounds)

    def __call__(self, x1_shard, x2=None, out=None, gather=False, M=None, on_gemm=None):
        """x2: [K, N] on rank src (ignored elsewhere).  out: optional [rows, N] result.
        on_gemm(p, fn): optional hook wrapping each panel GEMM launch (used for timing)."""
        from . import ext
        rows = x1_shard.shape[0]
        if out is None:
            out = x1_shard.new_empty(rows, self.N)
        if self.world == 1:
            def run():
                ext._matrix_mul(x1_shard, x2, out=out)
            (on_gemm(0, run) if on_gemm else run())
            return out
        if self.rank == self.src:
            if x2 is None or tuple(x2.shape) != (self.K, self.N):
                raise ValueError(f"rank {self.rank} is the source: x2 must be [{self.K}, {self.N}]")
        works = []
        for (n0, n1), buf in zip(self.bounds, self.bufs):
            # Pack panel p, then enqueue its broadcast (which waits for this pack only); the
            # next pack runs on the compute stream while the broadcast runs on NCCL's.
            if self.rank == self.src:
                buf.copy_(x2[:, n0:n1])
            works.append(dist.broadcast(buf, src=self.src, group=self.group, async_op=True))
        for p, ((n0, n1), buf, w) in enumerate(zip(self.bounds, self.bufs, works)):
            w.wait()

            def run(buf=buf, n0=n0, n1=n1):
                ext._matrix_mul(x1_shard, buf, out=out[:, n0:n1])
            (on_gemm(p, run) if on_gemm else run())
        if gather:
            if M is None:
                raise ValueError("gather=True needs the global row count M")
            return gather_rows(out, M, self.group)
        return out

    def run_host(self, h_x1_shard, h_x2=None, h_out=None, chunks=16, sync=True):
        """Host-buffer variant: x2 (rank src) and this rank's rows of x1 come from host memory
        and this rank's rows of C go back to it.  Row chunks of x1 stream through H2D -> GEMM
        (all panels) -> D2H with the three overlapping (tilec_b200.ext.pipelined_rows).  With
        several ranks, rank src copies x2's column panels straight from host memory into the
        panel buffers (one 2-D copy each, no packing) on the H2D stream, panel p just before
        x1's chunk p, and broadcasts each as soon as its copy is enqueued; a chunk's GEMM of
        panel p waits for broadcast p only."""
        from . import ext
        rows = h_x1_shard.shape[0]
        if h_out is None:
            h_out = torch.empty(rows, self.N, dtype=torch.float32, pin_memory=True)
        dev = self.device
        if self.rank == self.src and (h_x2 is None or tuple(h_x2.shape) != (self.K, self.N)):
            raise ValueError(f"rank {self.rank} is the source: h_x2 must be [{self.K}, {self.N}]")
        with torch.cuda.device(dev):
            if self.world == 1:
                d_x2 = torch.empty(self.K, self.N, dtype=torch.float32, device=dev)
                d_x2.copy_(h_x2, non_blocking=True)
                ext.pipelined_rows(h_x1_shard, h_out, dev, lambda d_x1, d_out: ext.chunk_compute(d_x1, d_x2),
                                   chunks=chunks, sync=sync)
                return h_out
            root = self.rank == self.src
            n_pan = len(self.bufs)
            works = [None] * n_pan
            if not root:
                # Enqueued before any H2D copy of this rank, so they wait for nothing local.
                works = broadcast_panels(self.bufs, self.src, self.group)
            staged = [0]

            def stage(i):
                # Rank src, on the H2D stream: panels up to p = i before x1's chunk i (all that
                # remain once the chunks are out), each broadcast right after its copy.
                if not root:
                    return
                upto = n_pan if i is None else min(n_pan, i + 1)
                while staged[0] < upto:
                    p = staged[0]
                    n0, n1 = self.bounds[p]
                    copy_columns_h2d(self.bufs[p], h_x2, n0, n1)
                    works[p] = dist.broadcast(self.bufs[p], src=self.src, group=self.group, async_op=True)
                    staged[0] += 1

            def make_compute(d_x1, d_out):
                parts = [((n0, n1), ext.chunk_compute(d_x1, buf)) for (n0, n1), buf in zip(self.bounds, self.bufs)]
                ready = [False] * n_pan

                def compute(a, c):
                    for p, ((n0, n1), fn) in enumerate(parts):
                        if not ready[p]:
                            works[p].wait()  # the compute stream waits for broadcast p
                            ready[p] = True
                        fn(a, c[:, n0:n1])
                return compute
            ext.pipelined_rows(h_x1_shard, h_out, dev, make_compute, chunks=chunks, sync=sync, h2d_hook=stage)
        return h_out


def matrix_mul_rowsharded(x1_shard, x2, group=None, src=0, gather=False, M=None, panels=2):
    """One-shot row-sharded matrix_mul (allocates panel buffers per call)."""
    K = x1_shard.shape[1]
    N = x2.shape[1] if x2 is not None else None
    if N is None:
        raise ValueError("every rank needs N: pass x2 (any [K, N] tensor on non-source ranks)")
    op = RowShardedMatmul(K, N, panels=panels, group=group, src=src, device=x1_shard.device)
    return op(x1_shard, x2, gather=gather, M=M)
