"""Row-sharded matrix_mul over NCCL on 2+ GPUs (run with -m gpu on a multi-GPU box).

Each rank is a child process on its own GPU.  Rank 0 owns x2 and broadcasts it in column
panels; every rank multiplies its row block of x1; the gathered result is checked against
an fp64 product on sampled rows and against a row-checksum identity.  Skipped when fewer
than two GPUs are visible.
"""
import datetime
import multiprocessing as mp
import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, M, K, N, panels, taper=False):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist
        from tilec_b200.dist import RowShardedMatmul, shard_rows
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        g = torch.Generator(device=dev).manual_seed(0)
        x1_full = torch.randn(M, K, device=dev, generator=g)   # same on every rank (same seed)
        x2_full = torch.randn(K, N, device=dev, generator=g) / K ** 0.5
        r0, r1 = shard_rows(M, world, rank)
        op = RowShardedMatmul(K, N, panels=panels, device=dev, taper=taper)
        x2 = x2_full if rank == 0 else None
        c_full = op(x1_full[r0:r1].contiguous(), x2, gather=True, M=M)
        torch.cuda.synchronize()
        # The host-buffer path on the same data gives the same rows: bit for bit, since every
        # row chunk runs the kernel and K split planned for the whole shard, except where that
        # plan is the pair kernel's stream-K form, which a row chunk (fewer tiles) cannot
        # reproduce; chunks then run one pair per tile, equal up to fp32 regrouping.
        from tilec_b200 import ext
        h_rows = op.run_host(x1_full[r0:r1].cpu().pin_memory(), x2_full.cpu().pin_memory() if rank == 0 else None,
                             chunks=3)
        shard = x1_full[r0:r1].contiguous()
        sk = any(ext.kernel_plan(shard, buf, detail=True)["stream_k"] for buf in op.bufs)
        d_rows = c_full[r0:r1].cpu()
        if sk:
            same = ((h_rows.double() - d_rows.double()).norm() / d_rows.double().norm()).item() <= 1e-5
        else:
            same = torch.equal(h_rows, d_rows)
        ok = True
        info = ""
        if rank == 0:
            rows = torch.unique(torch.linspace(0, M - 1, 24).round().long()).to(dev)
            ref = x1_full[rows].double() @ x2_full.double()
            err = ((c_full[rows].double() - ref).norm() / ref.norm()).item()
            rs = x1_full.double() @ x2_full.double().sum(1)
            err_rs = ((c_full.double().sum(1) - rs).norm() / rs.norm()).item()
            ok = err <= 1e-5 and err_rs <= 1e-5 and tuple(c_full.shape) == (M, N)
            info = f"rows relFrob {err:.2e}, checksum {err_rs:.2e}"
        ok = ok and same
        if not same:
            info += " host-path rows differ from device-path rows"
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok, info))
    except Exception:  # noqa: BLE001
        q.put((rank, False, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("M,K,N,panels,taper", [(8192, 2048, 4096, 2, False), (1001, 512, 777, 3, False),
                                               (65536 // 8, 8192, 8192, 2, False), (8192, 2048, 8192, 3, True)])
def test_rowsharded_two_gpus(M, K, N, panels, taper):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, M, K, N, panels, taper)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, ok, info = q.get(timeout=240)
            res[r] = (ok, info)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert res[r][0], f"rank {r}: {res[r][1]}"
