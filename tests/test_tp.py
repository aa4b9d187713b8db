"""Host logic of the tensor-parallel wrapper on CPU ranks (gloo, world size 2 and 3).

The local product is the oracle (numpy) here, so the test covers the sharding,
padding and all-gather reassembly; the GPU path runs the same wrapper with the
library GEMV and NCCL (tests/test_gpu_tp.py)."""
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
