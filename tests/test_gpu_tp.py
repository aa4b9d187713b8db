"""Tensor-parallel W4A16 GEMV over NCCL on two GPUs: each rank runs the library GEMV
on its row shard and the all-gathered output matches the oracle on the full matrix.
Skipped when fewer than two GPUs are visible."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, rows, cols, group, batch, q):
    import datetime

    import torch.distributed as dist

    import w4a16 as K
    from oracle import c_oracle
    from w4a16.tp import RowShardedW4A16, shard_rows

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator(device=dev).manual_seed(11)  # same weights on every rank
        w = (torch.randn(rows, cols, device=dev, generator=g) * 0.02).half()
        x = torch.randn(batch, cols, device=dev, generator=g).half()
        packed, scale = K.quantize_pack(w, group=group)
        tp = RowShardedW4A16(shard_rows(packed, world, rank), shard_rows(scale, world, rank), rows,
                             group=group)
        y = tp(x if batch > 1 else x[0])
        torch.cuda.synchronize()
        ref = c_oracle.gemv(packed.cpu().numpy(), scale.cpu().numpy(), x.cpu().numpy(), group=group)
        ref = ref[0] if batch == 1 else ref
        err = np.abs(y.cpu().numpy() - ref)
        ok = bool((err <= 1e-3 + 1e-3 * np.abs(ref)).all())
        q.put((rank, ok, float(err.max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("rows,cols,group,batch", [(128256, 2048, 128, 1), (14336, 4096, 128, 4),
                                                   (1000, 2048, 0, 1)])
def test_row_sharded_nccl(rows, cols, group, batch):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, rows, cols, group, batch, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, ok, err in res:
        assert ok, f"rank {rank}: max err {err}"


def _fused_worker(rank, world, port, rows, cols, group, out_dtype, q):
    import datetime

    import torch.distributed as dist

    import w4a16 as K
    from oracle import c_oracle
    from w4a16.tp import FusedAllGatherW4A16, shard_rows

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    tp = None
    try:
        g = torch.Generator(device=dev).manual_seed(12)  # same weights on every rank
        w = (torch.randn(rows, cols, device=dev, generator=g) * 0.02).half()
        xs = [torch.randn(cols, device=dev, generator=g).half() for _ in range(3)]
        packed, scale = K.quantize_pack(w, group=group)
        tp = FusedAllGatherW4A16(shard_rows(packed, world, rank), shard_rows(scale, world, rank), rows,
                                 group=group, out_dtype=out_dtype)
        pk, sc = packed.cpu().numpy(), scale.cpu().numpy()
        # references first: a rank must not stall between steps for longer than the
        # kernels' 2 s wait for their peers
        refs = [c_oracle.gemv(pk, sc, x.cpu().numpy(), group=group) for x in xs]
        dist.barrier()
        tol = 1e-3 if out_dtype == torch.float32 else 4e-3
        worst, ok = 0.0, True
        for step in range(6):  # consecutive steps with changing inputs reuse the same buffers
            y = tp(xs[step % 3], pdl=step % 2 == 1).clone()
            torch.cuda.synchronize()
            ref = refs[step % 3]
            err = np.abs(y.float().cpu().numpy() - ref)
            worst = max(worst, float(err.max()))
            ok &= bool((err <= tol + tol * np.abs(ref)).all())
        # captured in a CUDA graph: three steps per replay, the step flags advance on the device
        xg = xs[0].clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            tp(xg)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(3):  # chained: each step's start overlaps the previous one's tail
                tp(xg, pdl=True)
        for i in range(4):
            xg.copy_(xs[i % 3])
            graph.replay()
            torch.cuda.synchronize()
            ref = refs[i % 3]
            err = np.abs(tp.out.float().cpu().numpy() - ref)
            worst = max(worst, float(err.max()))
            ok &= bool((err <= tol + tol * np.abs(ref)).all())
        del graph
        ok &= K.read_device_error() == 0
        q.put((rank, ok, worst))
    finally:
        if tp is not None:
            tp.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("rows,cols,group,out_dtype", [(262144, 2048, 128, torch.float32),
                                                       (128256, 2048, 128, torch.float16),
                                                       (5000, 4096, 0, torch.float32)])
def test_fused_allgather(rows, cols, group, out_dtype):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, 2, port, rows, cols, group, out_dtype, q))
             for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, ok, err in res:
        assert ok, f"rank {rank}: max err {err}"
