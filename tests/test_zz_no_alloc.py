"""w4a16_gemv_noalloc: the split-K GEMV for callers that cannot allocate device memory.

Some runtimes fix their device memory plan at start-up, or expose an op interface
that passes only input and output buffers, so they cannot give the library a
workspace.  This entry point takes its split-K scratch from an array inside the
library instead.  The test calls it through the C ABI twice in a row (the second
call sees the array as the first left it) and compares each result with the
existing entry point w4a16_gemv run with its own workspace.  This file is collected
last so that a run stopping at the first failure has already run the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

import w4a16 as K
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
    for _ in range(2):
        y = _noalloc(packed, scale, x, group).cpu().numpy().astype(np.float64)
        err = np.abs(y - ref)
        assert (err <= ATOL + RTOL * np.abs(ref)).all(), f"max abs err {err.max():.3e}"


def test_noalloc_rejects_oversize_without_running():
    packed = torch.zeros(16, 4096, dtype=torch.uint8, device=DEV)
    scale = torch.ones(16, device=DEV)
    x = torch.zeros(8192, dtype=torch.float16, device=DEV)
    out = torch.full((16,), 7.0, device=DEV)
    # 600000 rows x 8192 columns would need ~19 MB of scratch: rejected on the host
    st = _lib.lib().w4a16_gemv_noalloc(_p(packed), _p(scale), 0, 0, _p(x), 600000, 8192, _p(out),
                                       None)
    assert st == -5  # W4A16_ERR_WORKSPACE
    assert b"static array" in _lib.lib().w4a16_last_error_string()
    torch.cuda.synchronize()
    assert (out == 7.0).all()
