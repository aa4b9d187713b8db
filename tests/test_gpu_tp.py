"""Tensor-parallel W4A16 GEMV over NCCL on two GPUs: each rank runs the library GEMV
on its row shard and the all-gathered output matches the oracle on the full matrix.
The multi-GPU tests are skipped when fewer than two GPUs are visible; the capacity
check of the fused all-gather runs on one GPU (it launches nothing)."""
import ctypes
import os
import socket
import time

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
        # the last step's stamps: every phase non-negative, the step well under a second
        tl = tp.timeline()
        ok &= all(v >= 0 for v in tl.values()) and 0 < tl["total"] < 1e6
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


# Llama-3-8B-shaped projections (hidden 4096, MLP 14336, GQA 32/8 heads of 128, vocab
# 128256): q, k (= v), gate (= up), down and the head, group-128 int4.
LLAMA8B_SHAPES = [("q_proj", 4096, 4096), ("kv_proj", 1024, 4096), ("gate_up", 14336, 4096),
                  ("down_proj", 4096, 14336), ("lm_head", 128256, 4096)]


def _llama8b_worker(rank, world, port, batches, q):
    import datetime

    import torch.distributed as dist

    import w4a16 as K
    from oracle import c_oracle
    from w4a16.tp import FusedAllGatherW4A16, RowShardedW4A16, shard_rows

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    results = []
    try:
        for name, rows, cols in LLAMA8B_SHAPES:
            g = torch.Generator(device=dev).manual_seed(rows + cols)  # same weights on every rank
            w = (torch.randn(rows, cols, device=dev, generator=g) * 0.02).half()
            packed, scale = K.quantize_pack(w, group=128)
            del w
            ps, ss = shard_rows(packed, world, rank), shard_rows(scale, world, rank)
            pk, sc = packed.cpu().numpy(), scale.cpu().numpy()
            xs = {b: torch.randn(b, cols, device=dev, generator=g).half() for b in batches}
            refs = {b: c_oracle.gemv(pk, sc, xs[b].cpu().numpy(), group=128) for b in batches}
            nccl = RowShardedW4A16(ps, ss, rows, group=128)
            for b in batches:
                y = nccl(xs[b] if b > 1 else xs[b][0])
                torch.cuda.synchronize()
                ref = refs[b] if b > 1 else refs[b][0]
                err = np.abs(y.cpu().numpy() - ref)
                results.append((name, b, "nccl", float(err.max()),
                                bool((err <= 1e-3 + 1e-3 * np.abs(ref)).all())))
            if 1 in batches:
                fused = FusedAllGatherW4A16(ps, ss, rows, group=128)
                try:
                    dist.barrier()
                    y = fused(xs[1][0], check=True).clone()
                    err = np.abs(y.cpu().numpy() - refs[1][0])
                    results.append((name, 1, "fused", float(err.max()),
                                    bool((err <= 1e-3 + 1e-3 * np.abs(refs[1][0])).all())))
                finally:
                    fused.close()
            del packed, scale, ps, ss
            torch.cuda.empty_cache()
        q.put((rank, results))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_llama8b_shapes_row_sharded_batches():
    """Every Llama-3-8B-shaped layer, batch 1, 4 and 16, row-sharded over two GPUs and
    gathered by NCCL (and, at batch 1, by the all-gather fused into the GEMV)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_llama8b_worker, args=(r, 2, port, (1, 4, 16), q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, cases in res:
        assert len(cases) == len(LLAMA8B_SHAPES) * 4
        for name, b, how, err, ok in cases:
            assert ok, f"rank {rank} {name} batch {b} ({how}): max err {err:.3e}"


def test_allgather_rejects_rows_outside_the_regions():
    """Rows that do not fit a region's gathered output are refused before any launch
    (two regions of one GPU stand in for two ranks; nothing runs, nothing waits)."""
    import w4a16 as K
    from w4a16 import _lib

    L = _lib.lib()
    torch.cuda.set_device(0)
    handle = ctypes.create_string_buffer(int(L.w4a16_tp_ipc_handle_bytes()))
    regions = []
    try:
        for _ in range(2):
            r = ctypes.c_void_p()
            assert L.w4a16_tp_region_alloc(4096 * 4, ctypes.byref(r), handle) == 0
            regions.append(r.value)
        arr = (ctypes.c_void_p * 2)(*regions)
        w = torch.randn(16, 256, device="cuda").half()
        packed, scale = K.quantize_pack(w, group=128)
        x = torch.randn(256, device="cuda").half()

        def call(row0, rows=16, odt=_lib.DTYPE_F32):
            return L.w4a16_gemv_allgather(ctypes.c_void_p(packed.data_ptr()), ctypes.c_void_p(scale.data_ptr()),
                                          0, 128, ctypes.c_void_p(x.data_ptr()), rows, 256, odt, row0, 0, 2,
                                          arr, None, 0, 0, None)

        assert call(4096 - 8) == -2                        # 8 rows past the end of 4096 fp32
        assert b"do not fit" in L.w4a16_last_error_string()
        assert call(1 << 40) == -2                         # far outside
        assert call(8192 - 8, odt=_lib.DTYPE_F16) == -2    # 16 KiB hold 8192 fp16 rows
        torch.cuda.synchronize()
        assert K.read_device_error() == 0                  # nothing ran
    finally:
        for r in regions:
            L.w4a16_tp_region_close(ctypes.c_void_p(r), 1)


def _missing_rank_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    import w4a16 as K
    from oracle import c_oracle
    from w4a16 import _lib
    from w4a16.tp import FusedAllGatherW4A16, shard_bounds, shard_rows

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    tp = None
    try:
        assert _lib.lib().w4a16_tp_set_peer_wait_ns(50 * 10**6) == 0   # 50 ms per wait
        rows, cols = 8192, 2048
        g = torch.Generator(device=dev).manual_seed(21)
        w = (torch.randn(rows, cols, device=dev, generator=g) * 0.02).half()
        xs = [torch.randn(cols, device=dev, generator=g).half() for _ in range(2)]
        packed, scale = K.quantize_pack(w, group=128)
        pk, sc = packed.cpu().numpy(), scale.cpu().numpy()
        refs = [c_oracle.gemv(pk, sc, x.cpu().numpy(), group=128) for x in xs]
        tp = FusedAllGatherW4A16(shard_rows(packed, world, rank), shard_rows(scale, world, rank), rows,
                                 group=128)
        lo, hi = shard_bounds(rows, world, rank)
        ok, info = True, {}
        for _ in range(2):  # both ranks take part: the whole output, no error
            dist.barrier()
            y = tp(xs[0], check=True).cpu().numpy()
            ok &= bool((np.abs(y - refs[0]) <= 1e-3 + 1e-3 * np.abs(refs[0])).all())
        dist.barrier()
        # rank 1 leaves out the next step (between steps, nothing in flight); rank 0 runs it
        if rank == 0:
            t0 = time.perf_counter()
            y = tp(xs[1]).cpu().numpy()   # returns once its waits for rank 1 ran out
            info["step_s"] = time.perf_counter() - t0
            info["code"] = tp.device_error()
            own = np.abs(y[lo:hi] - refs[1][lo:hi])
            info["own_rows_ok"] = bool((own <= 1e-3 + 1e-3 * np.abs(refs[1][lo:hi])).all())
        else:
            info["code"] = tp.device_error()
        dist.barrier()
        assert _lib.lib().w4a16_tp_set_peer_wait_ns(0) == 0
        q.put((rank, ok, info))
    finally:
        if tp is not None:
            tp.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_allgather_missing_rank_times_out():
    """A rank that skips a step: the other rank's call still returns (its waits give up
    after the 50 ms limit), the device error word reads 2, and its own rows are right."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_missing_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (ok, info)) for r, ok, info in (q.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0][0] and res[1][0], "the steps with both ranks were wrong"
    info0, info1 = res[0][1], res[1][1]
    assert info0["code"] == 2, info0
    assert info0["own_rows_ok"], info0
    assert info0["step_s"] < 5.0, info0
    assert info1["code"] == 0, info1
