"""Tensor-parallel W4A16 GEMV: weights sharded by output rows, outputs all-gathered.

No counterpart in the reference (it is single-GPU only).  Rank r of P holds rows
[r*N/P, (r+1)*N/P) of `packed` and of `scale` (group-128 scale rows travel with
their weight rows); the activation is replicated.  Each rank runs the local
sm_100a GEMV into its slice of a [batch, N] buffer and one all_gather_into_tensor
over NCCL (NVLink / NVSwitch) assembles the full output on every rank.  The row
split is the only exchange: no partial sums cross GPUs.

Shard boundaries are rounded to multiples of 16 rows (the kernel's tile) so that
every rank's slice starts on a tile; the last rank takes the remainder.
"""
import torch
import torch.distributed as dist

ROW_ALIGN = 16


def shard_bounds(rows, world, rank, align=ROW_ALIGN):
    """[lo, hi) rows owned by `rank`; shards are multiples of `align` except the last."""
    per = -(-rows // world)               # ceil
    per = -(-per // align) * align        # round up to the alignment
    lo = min(rank * per, rows)
    hi = min(lo + per, rows)
    return lo, hi


def shard_rows(t, world, rank, align=ROW_ALIGN):
    """The rows of `t` (packed [N, K/2] or scale [N] / [N, G]) that `rank` owns."""
    lo, hi = shard_bounds(t.shape[0], world, rank, align)
    return t[lo:hi].contiguous()


class RowShardedW4A16:
    """One row shard of an int4 weight and the all-gather that reassembles outputs.

    packed_shard / scale_shard: this rank's rows (see shard_rows); rows: the full N.
    gemv_fn(packed, scale, x, out) computes the local product into `out`; the
    default is the library's GEMV.  A CPU-testable seam: tests pass a torch matmul.
    """

    def __init__(self, packed_shard, scale_shard, rows, group=0, process_group=None,
                 gemv_fn=None, out_dtype=torch.float32):
        self.pg = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        self.rows = rows
        self.group = group
        self.packed = packed_shard
        self.scale = scale_shard
        self.out_dtype = out_dtype
        lo, hi = shard_bounds(rows, self.world, self.rank)
        if packed_shard.shape[0] != hi - lo:
            raise ValueError(f"rank {self.rank} owns rows [{lo},{hi}) but got {packed_shard.shape[0]}")
        # all_gather_into_tensor needs equal-sized chunks: pad every shard to the largest
        self.chunk = shard_bounds(rows, self.world, 0)[1]
        self.gemv_fn = gemv_fn or self._library_gemv

    def _library_gemv(self, packed, scale, x, out):
        from . import kernels as K

        return K.gemv(packed, scale, x, group=self.group, out=out, out_dtype=out.dtype)

    def __call__(self, x, out=None):
        """x: [K] or [batch, K] (fp16, replicated).  Returns [N] or [batch, N] on every rank."""
        batch = 1 if x.dim() == 1 else x.shape[0]
        dev = x.device
        n = self.packed.shape[0]
        local = torch.empty((batch, self.chunk), dtype=self.out_dtype, device=dev)
        if n:
            xx = x if x.dim() == 2 else x.view(1, -1)
            if n == self.chunk:
                self.gemv_fn(self.packed, self.scale, xx, local)
            else:
                res = torch.empty((batch, n), dtype=self.out_dtype, device=dev)
                self.gemv_fn(self.packed, self.scale, xx, res)
                local[:, :n].copy_(res)
        gathered = torch.empty((self.world, batch, self.chunk), dtype=self.out_dtype, device=dev)
        dist.all_gather_into_tensor(gathered.view(-1), local.view(-1), group=self.pg)
        if batch == 1 and self.chunk * self.world == self.rows and out is None:
            # equal shards: the gathered buffer already is the output, in row order
            full = gathered.view(1, self.rows)
            return full.view(-1) if x.dim() == 1 else full
        full = torch.empty((batch, self.rows), dtype=self.out_dtype, device=dev) if out is None else out.view(batch, self.rows)
        for r in range(self.world):
            lo, hi = shard_bounds(self.rows, self.world, r)
            if hi > lo:
                full[:, lo:hi] = gathered[r, :, : hi - lo]
        return full.view(-1) if x.dim() == 1 and out is None else full
