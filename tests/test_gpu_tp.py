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
