"""Host logic of the tensor-parallel wrapper on CPU ranks (gloo, world size 2 and 3).

The local product is the oracle (numpy) here, so the test covers the sharding,
padding and all-gather reassembly; the GPU path runs the same wrapper with the
library GEMV and NCCL (tests/test_gpu_tp.py)."""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import w4a16_oracle as O
from w4a16.tp import RowShardedW4A16, shard_bounds, shard_rows


def test_shard_bounds_cover_rows_in_order():
    for rows in (1, 15, 16, 17, 100, 128256, 262144):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(rows, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == rows
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c and a <= b
            for lo, hi in spans:
                assert lo % 16 == 0 or lo == rows  # every shard starts on a 16-row tile


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, rows, cols, group, batch, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        qc, s = O.quantize_int4_group(w, group) if group else O.quantize_int4_symmetric(w)
        packed = torch.from_numpy(O.pack_int4_interleaved(qc))
        scale = torch.from_numpy(s)
        x = torch.from_numpy(rng.standard_normal((batch, cols)).astype(np.float16))

        def oracle_gemv(p_, s_, x_, out):
            out.copy_(torch.from_numpy(O.gemv_packed(p_.numpy(), s_.numpy(), x_.numpy(), group)))

        tp = RowShardedW4A16(shard_rows(packed, world, rank), shard_rows(scale, world, rank), rows,
                             group=group, gemv_fn=oracle_gemv)
        y = tp(x if batch > 1 else x[0])
        ref = O.gemv(qc, s, x if batch > 1 else x[0], group)
        q.put((rank, float(np.abs(y.double().numpy() - ref).max()), tuple(y.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,rows,cols,group,batch", [
    (2, 512, 256, 0, 1), (2, 500, 256, 128, 1), (3, 100, 128, 128, 3), (2, 64, 512, 0, 4)])
def test_row_sharded_gather_matches_full_product(world, rows, cols, group, batch):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, rows, cols, group, batch, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want_shape = (rows,) if batch == 1 else (batch, rows)
    for rank, err, shape in results:
        assert shape == want_shape
        assert err < 1e-5, f"rank {rank}: max err {err}"


class _FakeTpLib:
    """Stands in for the library's region / IPC / launch calls on CPU ranks."""

    def __init__(self, rank):
        self.rank = rank
        self.opened, self.closed, self.launches = [], [], []

    def w4a16_tp_ipc_handle_bytes(self):
        return 64

    def w4a16_tp_header_bytes(self):
        return 256

    def w4a16_tp_region_alloc(self, nbytes, pptr, handle):
        pptr._obj.value = (self.rank + 1) << 20
        tag = f"region-of-rank-{self.rank}-{nbytes}".encode()
        ctypes.memmove(handle, tag.ljust(64, b"\0"), 64)
        return 0

    def w4a16_tp_region_open(self, handle, pptr):
        text = handle.raw.rstrip(b"\0").decode()
        self.opened.append(text)
        pptr._obj.value = (int(text.split("-")[3]) + 1) << 20
        return 0

    def w4a16_tp_region_close(self, ptr, owned):
        self.closed.append((ptr.value, owned))
        return 0

    def w4a16_gemv_allgather(self, packed, scale, sdt, group, x, rows, cols, odt, row0, rank, nranks,
                             regions, ws, wsb, flags, stream):
        self.launches.append((rows, cols, row0, rank, nranks, [regions[k] for k in range(nranks)]))
        return 0


def _fused_host_worker(rank, world, port, rows, q):
    from w4a16.tp import FusedAllGatherW4A16

    class CpuFused(FusedAllGatherW4A16):
        def _make_out(self, ptr, n, dtype):
            self.out_ptr = ptr
            return torch.zeros(n, dtype=dtype)

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lib = _FakeTpLib(rank)
        lo, hi = shard_bounds(rows, world, rank)
        packed = torch.zeros(hi - lo, 128, dtype=torch.uint8)
        scale = torch.ones(hi - lo, 2)
        tp = CpuFused(packed, scale, rows, group=128, lib=lib)
        tp.launch(packed, scale, torch.zeros(256, dtype=torch.float16), stream=ctypes.c_void_p(0))
        tp.close()
        q.put((rank, tp.regions, lib.opened, lib.launches, lib.closed, tp.out_ptr, (lo, hi)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,rows", [(2, 1000), (3, 4096)])
def test_fused_allgather_host_logic(world, rows):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_host_worker, args=(r, world, port, rows, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=120) for _ in range(world)])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [(k + 1) << 20 for k in range(world)]
    for rank, regions, opened, launches, closed, out_ptr, (lo, hi) in results:
        assert regions == want                                  # every rank's region, in rank order
        assert sorted(opened) == sorted(f"region-of-rank-{k}-{rows * 4}" for k in range(world) if k != rank)
        assert launches == [(hi - lo, 256, lo, rank, world, want)]
        assert out_ptr == want[rank] + 256                      # output after the header
        assert sorted(closed) == sorted([(w, 0) for k, w in enumerate(want) if k != rank] + [(want[rank], 1)])


# Llama-3-8B-shaped projections (q, k = v, gate = up, down, head), group-128
LLAMA8B_SHAPES = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]


def _llama8b_worker(rank, world, port, q):
    from oracle import c_oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        threads = max(1, (os.cpu_count() or 2) // world)
        out = []
        for rows, cols in LLAMA8B_SHAPES:
            rng = np.random.default_rng(rows + cols)   # the same matrix on every rank
            packed = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
            scale = (rng.random((rows, cols // 128), dtype=np.float32) * 2e-3 + 2e-3)
            for batch in (1, 4, 16):
                if rows == 128256 and batch == 4:
                    continue  # the head at batch 1 and 16 is enough here
                x = rng.standard_normal((batch, cols)).astype(np.float16)

                def local_gemv(p_, s_, x_, res):
                    res.copy_(torch.from_numpy(c_oracle.gemv(p_.numpy(), s_.numpy(), x_.numpy(), group=128,
                                                             threads=threads)))

                tp = RowShardedW4A16(shard_rows(torch.from_numpy(packed), world, rank),
                                     shard_rows(torch.from_numpy(scale), world, rank), rows, group=128,
                                     gemv_fn=local_gemv)
                y = tp(torch.from_numpy(x if batch > 1 else x[0]))
                ref = c_oracle.gemv(packed, scale, x, group=128, threads=threads)
                ref = ref if batch > 1 else ref[0]
                out.append((rows, cols, batch, tuple(y.shape), float(np.abs(y.numpy() - ref).max())))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_llama8b_shapes_row_sharded_gather(world):
    """The Llama-3-8B-shaped layers at batch 1, 4 and 16 sharded over 2 and 3 CPU ranks:
    the gathered output equals the product over the whole matrix (same summation per row)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_llama8b_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, cases in results:
        assert len(cases) == 14
        for rows, cols, batch, shape, err in cases:
            assert shape == ((rows,) if batch == 1 else (batch, rows))
            assert err == 0.0, f"rank {rank} {rows}x{cols} batch {batch}: max err {err}"
