"""Row-sharding logic of tilec_b200.dist on CPU ranks (gloo, world size 2).

The GEMM itself needs a GPU; here the partition, the panel packing, the panel
broadcast from the source rank, the row gather and the failure paths run on CPU ranks,
with the per-rank product computed by the test itself.
"""
import datetime
import multiprocessing as mp
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist

from tilec_b200.dist import gather_rows, pack_panels, panel_bounds, broadcast_panels, shard_rows


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _worker_rowsharded(rank, world, port, q):
    try:
        _init(rank, world, port)
        M, K, N = 37, 16, 300
        g = torch.Generator().manual_seed(0)
        x1 = torch.randn(M, K, generator=g)
        x2 = torch.randn(K, N, generator=g)
        r0, r1 = shard_rows(M, world, rank)
        bounds = panel_bounds(N, 2, align=128)
        bufs = [torch.empty(K, n1 - n0) for n0, n1 in bounds]
        if rank == 0:
            pack_panels(x2, bounds, bufs)
        works = broadcast_panels(bufs, src=0)
        out = torch.empty(r1 - r0, N)
        for (n0, n1), b, w in zip(bounds, bufs, works):
            w.wait()
            assert torch.equal(b, x2[:, n0:n1])
            out[:, n0:n1] = x1[r0:r1].double().matmul(b.double()).float()
        full = gather_rows(out, M)
        ref = x1.double().matmul(x2.double()).float()
        q.put((rank, bool(torch.equal(full, ref)), None))
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        q.put((rank, False, traceback.format_exc()))


def _worker_missing_rank(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=3)
        if rank == 1:
            q.put((rank, True, None))  # leaves without joining the broadcast
            return
        buf = torch.zeros(4, 4)
        try:
            dist.broadcast(buf, src=0, async_op=True).wait()
            dist.broadcast(buf, src=1, async_op=True).wait()
            q.put((rank, False, "collective with a missing rank returned"))
        except RuntimeError as e:
            q.put((rank, True, str(e)[:200]))
    except Exception:  # noqa: BLE001
        q.put((rank, False, traceback.format_exc()))


def _run(target, world=2, timeout=90):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, ok, info = q.get(timeout=timeout)
            results[rank] = (ok, info)
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    return results


def test_shard_rows_partition():
    for M in (0, 1, 7, 65536, 65537):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_rows(M, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == M
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    assert shard_rows(65536, 8, 3) == (24576, 32768)
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def test_panel_bounds():
    assert panel_bounds(8192, 2) == [(0, 4096), (4096, 8192)]
    assert panel_bounds(8192, 1) == [(0, 8192)]
    # widths round up to the alignment, so fewer panels than asked may come back
    assert panel_bounds(777, 3, align=256) == [(0, 512), (512, 777)]
    b = panel_bounds(1000, 3, align=128)
    assert b == [(0, 384), (384, 768), (768, 1000)]
    assert all(n1 > n0 for n0, n1 in b)
    assert panel_bounds(0, 4) == []
    # tapered: shares 1, 2, 4, ... of N, each rounded up to the alignment; contiguous cover
    assert panel_bounds(8192, 3, taper=True) == [(0, 1280), (1280, 3584), (3584, 8192)]
    assert panel_bounds(8192, 4, taper=True) == [(0, 768), (768, 1792), (1792, 3840), (3840, 8192)]
    assert panel_bounds(8192, 1, taper=True) == [(0, 8192)]
    assert panel_bounds(300, 4, taper=True) == [(0, 256), (256, 300)]
    for n in (1, 255, 777, 1000, 4097, 8192):
        for p in (2, 3, 5):
            b = panel_bounds(n, p, taper=True)
            assert b[0][0] == 0 and b[-1][1] == n and all(x[1] == y[0] for x, y in zip(b, b[1:]))
            assert all(n1 > n0 for n0, n1 in b) and all((n1 - n0) % 256 == 0 for n0, n1 in b[:-1])


def test_rowsharded_broadcast_and_gather_gloo():
    res = _run(_worker_rowsharded)
    for rank, (ok, info) in sorted(res.items()):
        assert ok, f"rank {rank}: {info}"


def test_missing_rank_times_out_with_error():
    res = _run(_worker_missing_rank)
    ok, info = res[0]
    assert ok, info
