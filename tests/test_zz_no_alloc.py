"""w4a16_gemv_noalloc: the split-K GEMV for callers that cannot allocate device memory.

Some runtimes fix their device memory plan at start-up, or expose an op interface
that passes only input and output buffers, so they cannot give the library a
workspace.  This entry point takes its split-K scratch from an array inside the
library instead.  The test calls it through the C ABI twice in a row (the second
call sees the array as the first left it) and compares each result with the
existing entry point w4a16_gemv run with its own workspace, and with the oracle.
This file is collected last so that a run stopping at the first failure has already
run the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

import w4a16 as K
from oracle import c_oracle
from w4a16 import _lib

pytestmark = pytest.mark.gpu

ATOL = RTOL = 1e-3
DEV = "cuda"


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc(packed, scale, x, group):
    rows, cols = packed.shape[0], packed.shape[1] * 2
    out = torch.empty(rows, dtype=torch.float32, device=DEV)
    sdt = _lib.DTYPE_F32 if scale.dtype == torch.float32 else _lib.DTYPE_F16
    st = _lib.lib().w4a16_gemv_noalloc(_p(packed), _p(scale), sdt, group, _p(x), rows, cols, _p(out),
                                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, _lib.lib().w4a16_last_error_string()
    return out


CASES = [(2048, 8192, 128, torch.float32), (8192, 2048, 0, torch.float32),
         (3000, 4096, 128, torch.float16), (1000, 11008, 0, torch.float32)]


@pytest.mark.parametrize("rows,cols,group,sdt", CASES,
                         ids=[f"{r}x{c}-g{g}-{str(d)[-7:]}" for r, c, g, d in CASES])
def test_noalloc_matches_workspace_entry_two_calls(rows, cols, group, sdt):
    g = torch.Generator(device=DEV).manual_seed(rows + cols)
    w = (torch.randn(rows, cols, device=DEV, generator=g) * 0.02).half()
    x = torch.randn(cols, device=DEV, generator=g).half()
    packed, scale = K.quantize_pack(w, group=group, scale_dtype=sdt)
    ref = K.gemv(packed, scale, x, group=group).cpu().numpy().astype(np.float64)
    oracle = c_oracle.gemv(packed.cpu().numpy(), scale.float().cpu().numpy(), x.cpu().numpy(),
                           group=group).astype(np.float64)
    for _ in range(2):
        y = _noalloc(packed, scale, x, group).cpu().numpy().astype(np.float64)
        err = np.abs(y - ref)
        assert (err <= ATOL + RTOL * np.abs(ref)).all(), f"max abs err {err.max():.3e}"
        err = np.abs(y - oracle)
        assert (err <= ATOL + RTOL * np.abs(oracle)).all(), f"max abs err vs oracle {err.max():.3e}"


def test_noalloc_scratch_does_not_grow_with_the_matrix():
    # the scratch need is set by the warp count, not by rows x cols: the largest
    # shape of the benchmark runs through the static array as well
    L = _lib.lib()
    assert L.w4a16_gemv_workspace_bytes(1, 262144, 2048) == L.w4a16_gemv_workspace_bytes(1, 2048, 8192)
    assert L.w4a16_gemv_workspace_bytes(1, 262144, 2048) <= 4 << 20
    g = torch.Generator(device=DEV).manual_seed(5)
    w = (torch.randn(262144, 2048, device=DEV, generator=g) * 0.02).half()
    x = torch.randn(2048, device=DEV, generator=g).half()
    packed, scale = K.quantize_pack(w, group=128)
    del w
    ref = K.gemv(packed, scale, x, group=128).cpu().numpy().astype(np.float64)
    for _ in range(2):
        y = _noalloc(packed, scale, x, 128).cpu().numpy().astype(np.float64)
        err = np.abs(y - ref)
        assert (err <= ATOL + RTOL * np.abs(ref)).all(), f"max abs err {err.max():.3e}"
