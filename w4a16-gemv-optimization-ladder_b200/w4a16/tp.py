"""Tensor-parallel W4A16 GEMV: weights sharded by output rows, outputs all-gathered.

No counterpart in the reference (it is single-GPU only).  Rank r of P holds rows
[r*N/P, (r+1)*N/P) of `packed` and of `scale` (group-128 scale rows travel with
their weight rows); the activation is replicated.  Each rank runs the local
sm_100a GEMV into its slice of a [batch, N] buffer and one all_gather_into_tensor
over NCCL (NVLink / NVSwitch) assembles the full output on every rank.  The row
split is the only exchange: no partial sums cross GPUs.

Shard boundaries are rounded to multiples of 16 rows (the kernel's tile) so that
every rank's slice starts on a tile; the last rank takes the remainder.

FusedAllGatherW4A16 does the same for one activation vector without NCCL: the GEMV's
epilogue stores each output row into every rank's gathered buffer through NVLink
(CUDA IPC mappings of the peers' buffers), with step flags in the same buffers.
"""
import ctypes

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


class _DeviceArray:
    """A raw device allocation seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr, n, dtype):
        typestr = {torch.float32: "<f4", torch.float16: "<f2"}[dtype]
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class FusedAllGatherW4A16:
    """Row shard of an int4 weight whose GEMV writes straight into every rank's output.

    Each rank allocates one region (header + the full [rows] output) with the library,
    shares its CUDA IPC handle over `process_group`, and opens the other ranks' regions;
    __call__(x) then runs w4a16_gemv_allgather: this rank's rows land in all ranks'
    outputs, and the call returns when (on the stream) every rank has finished the step.
    The returned tensor is the same buffer every call (valid until the next call).
    One activation vector (fp16 [K]); 2..8 ranks; interleaved packing.
    """

    def __init__(self, packed_shard, scale_shard, rows, group=0, process_group=None,
                 out_dtype=torch.float32, lib=None):
        from . import _lib
        from . import kernels as K

        self.pg = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        if not 2 <= self.world <= 8:
            raise ValueError(f"the fused all-gather takes 2..8 ranks, got {self.world}")
        self.rows, self.group, self.out_dtype = rows, group, out_dtype
        self.packed, self.scale = packed_shard, scale_shard
        self.lo, self.hi = shard_bounds(rows, self.world, self.rank)
        if packed_shard.shape[0] != self.hi - self.lo or self.hi <= self.lo:
            raise ValueError(f"rank {self.rank} owns rows [{self.lo},{self.hi}) but got {packed_shard.shape[0]}")
        self._check = _lib.check
        self.lib = lib or _lib.lib()
        esize = 4 if out_dtype == torch.float32 else 2
        self._odt = _lib.DTYPE_F32 if out_dtype == torch.float32 else _lib.DTYPE_F16
        handle = ctypes.create_string_buffer(int(self.lib.w4a16_tp_ipc_handle_bytes()))
        mine = ctypes.c_void_p()
        self._check(self.lib.w4a16_tp_region_alloc(rows * esize, ctypes.byref(mine), handle),
                    "w4a16_tp_region_alloc")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=process_group)
        self.regions = []
        for k, h in enumerate(handles):
            if k == self.rank:
                self.regions.append(mine.value)
                continue
            ptr = ctypes.c_void_p()
            self._check(self.lib.w4a16_tp_region_open(ctypes.create_string_buffer(h, len(h)),
                                                       ctypes.byref(ptr)), "w4a16_tp_region_open")
            self.regions.append(ptr.value)
        self._regions = (ctypes.c_void_p * self.world)(*self.regions)
        dist.barrier(group=process_group)  # every rank holds every mapping before the first step
        self.device = packed_shard.device
        self.out = self._make_out(mine.value + int(self.lib.w4a16_tp_header_bytes()), rows, out_dtype)
        # two split-K workspaces: chained (pdl) launches overlap neighbours, which must not share one
        self.workspaces = [K.new_workspace(self.device) for _ in range(2)] if self.device.type == "cuda" else None
        self._step = 0
        self._closed = False

    def _make_out(self, ptr, n, dtype):
        return torch.as_tensor(_DeviceArray(ptr, n, dtype), device=self.device)

    def launch(self, packed, scale, x, stream=None, pdl=False, check=False):
        """One step with explicit weights (this rank's rows), for callers that alternate
        several weight copies of the same shape.  pdl: chain to the previous kernel on the
        stream (programmatic dependent launch); the workspaces alternate per call.
        check: wait for the step and raise if a wait on another rank ran out (see
        device_error); without it the step stays asynchronous."""
        from . import _lib
        from . import kernels as K

        s = stream if stream is not None else K._stream(self.device)
        ws = self.workspaces[self._step % 2] if self.workspaces is not None else None
        self._step += 1
        st = self.lib.w4a16_gemv_allgather(
            ctypes.c_void_p(packed.data_ptr()), ctypes.c_void_p(scale.data_ptr()),
            0 if scale.dtype == torch.float32 else 1, self.group, ctypes.c_void_p(x.data_ptr()),
            packed.shape[0], packed.shape[1] * 2, self._odt, self.lo, self.rank, self.world,
            self._regions, ctypes.c_void_p(ws.data_ptr()) if ws is not None else None,
            ws.numel() if ws is not None else 0, _lib.LAUNCH_PDL if pdl else 0, s)
        self._check(st, "w4a16_gemv_allgather")
        if check:
            code = self.device_error(stream=s)
            if code:
                raise RuntimeError(f"w4a16_gemv_allgather: device error {code} (a rank's flags did not "
                                   "arrive in time; only this rank's rows of the output are current)")
        return self.out

    def device_error(self, stream=None):
        """Read and clear the device error word after the steps issued so far (synchronises
        the stream): 0 = every step assembled the whole output; 2 = a wait on another rank
        ran out, and that step wrote only this rank's rows.  After a non-zero code the
        ranks' step numbers disagree: close this object and build a new one.  The split-K
        workspaces are zero-filled again, as a warp that gave up may have left counters."""
        from . import _lib
        from . import kernels as K

        s = stream if stream is not None else K._stream(self.device)
        code = ctypes.c_int(0)
        with torch.cuda.device(self.device):
            self._check(self.lib.w4a16_read_device_error(ctypes.byref(code), s), "w4a16_read_device_error")
            if code.value and self.workspaces is not None:
                for w in self.workspaces:
                    w.zero_()
        return code.value

    def timeline(self, stream=None):
        """The last step on this rank, from the %globaltimer stamps its kernel wrote into this
        rank's region (synchronises the stream), in µs: `start_wait` from publishing this
        rank's start flags until the first warp of the first CTA, about to store its first
        tile, has seen every rank's start flag (so at least that tile's compute); `to_done`
        from there until every CTA's rows are stored and fenced; `done_wait` until every
        rank's done flag is seen; `total` the sum."""
        from . import kernels as K

        s = stream if stream is not None else K._stream(self.device)
        t = (ctypes.c_ulonglong * 4)()
        with torch.cuda.device(self.device):
            self._check(self.lib.w4a16_tp_region_timeline(ctypes.c_void_p(self.regions[self.rank]), t, s),
                        "w4a16_tp_region_timeline")
        t0, t1, t2, t3 = (int(v) for v in t)
        return {"start_wait": (t1 - t0) / 1e3, "to_done": (t2 - t1) / 1e3, "done_wait": (t3 - t2) / 1e3,
                "total": (t3 - t0) / 1e3}

    def __call__(self, x, pdl=False, check=False):
        if not (isinstance(x, torch.Tensor) and x.dtype == torch.float16 and x.dim() == 1
                and x.is_contiguous() and x.shape[0] == self.packed.shape[1] * 2 and x.device == self.device):
            raise RuntimeError("x must be a contiguous fp16 [cols] tensor on this rank's device")
        with torch.cuda.device(self.device):
            return self.launch(self.packed, self.scale, x, pdl=pdl, check=check)

    def close(self):
        """Unmap the peers' regions and free this rank's (after every rank is done)."""
        if self._closed:
            return
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.pg)
        for k, ptr in enumerate(self.regions):
            if k != self.rank:
                self.lib.w4a16_tp_region_close(ctypes.c_void_p(ptr), 0)
        dist.barrier(group=self.pg)
        self.lib.w4a16_tp_region_close(ctypes.c_void_p(self.regions[self.rank]), 1)
        self._closed = True
