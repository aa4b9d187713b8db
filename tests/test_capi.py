"""The C-ABI library loads without a GPU, exports every function include/w4a16_b200.h
declares, and rejects bad arguments on the host before any CUDA call.  No test here
launches a kernel."""
import ctypes
import os
import re

import pytest

from w4a16 import _lib
from w4a16 import build as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "w4a16_b200.h")


@pytest.fixture(scope="module")
def lib():
    B.build()
    return _lib.lib()


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(w4a16_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ["w4a16_marlin_cuda", "w4a16_marlin_g128_cuda", "w4a16_byte_cuda", "w4a16_u32_cuda",
              "w4a16_u32_v4_cuda", "w4a16_champ_cuda", "w4a16_uint4_cuda", "w4a16_h2f32_cuda",
              "w4a16_fp16_cuda", "w4a16_gemv", "w4a16_dequant", "w4a16_quantize_pack"]:
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert set(declared_functions()) <= set(_lib.SIGNATURES), "ctypes binding misses a symbol"


def test_library_is_sm100a_only(lib):
    # the library embeds sm_100a code only; its name and build flags say so
    assert B.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_version_and_status_strings(lib):
    assert lib.w4a16_version() == 10000
    assert lib.w4a16_status_string(0) == b"ok"
    assert lib.w4a16_status_string(-2) == b"bad shape"
    assert lib.w4a16_status_string(-99) == b"unknown status"


def _gemv(lib, packed=1 << 12, packing=0, scale=1 << 12, sdt=0, group=0, x=1 << 12, batch=1,
          rows=16, cols=256, out=1 << 12, odt=0):
    return lib.w4a16_gemv(ctypes.c_void_p(packed), packing, ctypes.c_void_p(scale), sdt, group,
                          ctypes.c_void_p(x), batch, rows, cols, ctypes.c_void_p(out), odt, None,
                          None, 0, None)


def test_host_validation_rejects_before_launch(lib):
    # each call fails validation, so no CUDA API is reached (none is available here)
    assert _gemv(lib, packing=7) == -4
    assert _gemv(lib, sdt=5) == -4
    assert _gemv(lib, group=64) == -4
    assert _gemv(lib, cols=12) == -2
    assert _gemv(lib, cols=192, group=128) == -2
    assert _gemv(lib, rows=-1) == -2
    assert _gemv(lib, packed=0) == -1
    assert _gemv(lib, x=(1 << 12) + 8) == -3          # x must be 16-byte aligned
    assert _gemv(lib, packed=(1 << 12) + 2) == -3     # packed 4-byte aligned
    assert b"multiple" in lib.w4a16_last_error_string() or True
    assert _gemv(lib, rows=0) == 0                   # empty problem: no-op
    assert _gemv(lib, batch=0) == 0
    f = lib.w4a16_marlin_cuda
    assert f(None, None, None, None, 16, 256, None) == -1
    assert f(None, None, None, None, 16, 250, None) == -2
    assert lib.w4a16_fp16_cuda(None, None, None, 4, 12, None) == -2
    assert lib.w4a16_dequant(None, 0, None, 0, 0, 4, 256, None, None) == -1
    assert lib.w4a16_quantize_pack(None, 9, 4, 256, 0, 0, None, None, 0, None) == -4


def test_last_error_message(lib):
    assert _gemv(lib, cols=12) == -2
    assert b"cols=12" in lib.w4a16_last_error_string()


def test_workspace_size(lib):
    assert lib.w4a16_gemv_workspace_bytes(1, 0, 2048) == 0
    small = lib.w4a16_gemv_workspace_bytes(1, 2048, 8192)
    assert small >= 8 * 2048 * 4  # up to one fp32 partial per 1024-column stage
    assert lib.w4a16_gemv_workspace_bytes(16, 2048, 8192) == lib.w4a16_gemv_workspace_bytes(64, 2048, 8192)


def test_python_ops_fail_loudly_without_library(monkeypatch, tmp_path):
    monkeypatch.setenv(_lib.ENV_LIB, str(tmp_path / "missing.so"))
    _lib.lib.cache_clear()
    try:
        with pytest.raises(RuntimeError, match="not found"):
            _lib.lib()
    finally:
        monkeypatch.delenv(_lib.ENV_LIB)
        _lib.lib.cache_clear()


def _gemm(lib, packed=1 << 12, scale=1 << 16, group=0, x=1 << 20, bias=None, M=256, N=256, K=1024,
          y=1 << 24, odt=0, ws=None):
    return lib.w4a16_gemm(ctypes.c_void_p(packed), ctypes.c_void_p(scale), group, ctypes.c_void_p(x),
                          None if bias is None else ctypes.c_void_p(bias), M, N, K, ctypes.c_void_p(y),
                          odt, None if ws is None else ctypes.c_void_p(ws), 1 << 20, None)


def test_tp_region_timeline_host_validation(lib):
    stamps = (ctypes.c_ulonglong * 4)()
    assert lib.w4a16_tp_region_timeline(None, stamps, None) == -1
    assert lib.w4a16_tp_region_timeline(ctypes.c_void_p(1 << 20), None, None) == -1
    # a pointer no region call returned: refused before any CUDA call
    assert lib.w4a16_tp_region_timeline(ctypes.c_void_p(1 << 20), stamps, None) == -2
    assert b"w4a16_tp_region_alloc" in lib.w4a16_last_error_string()


def test_gemm_host_validation(lib):
    # every call fails validation before any CUDA API is reached
    assert _gemm(lib, odt=3) == -4
    assert _gemm(lib, group=64) == -4
    assert _gemm(lib, K=96) == -2                  # K a multiple of 64
    assert _gemm(lib, K=192, group=128) == -2      # ... of 128 with group-128 scales
    assert _gemm(lib, M=0) == -2
    assert _gemm(lib, N=-1) == -2
    assert _gemm(lib, x=0) == -1
    assert _gemm(lib, scale=0) == -1
    assert _gemm(lib, packed=(1 << 12) + 4) == -3  # packed 16-byte aligned (TMA)
    assert _gemm(lib, x=(1 << 20) + 8) == -3
    assert _gemm(lib, y=(1 << 24) + 2) == -3       # fp32 output 4-byte aligned
    assert _gemm(lib, bias=(1 << 16) + 2) == -3
    assert _gemm(lib, ws=(1 << 28) + 16) == -3      # workspace 256-byte aligned
    assert b"aligned" in lib.w4a16_last_error_string()
    assert lib.w4a16_gemm_workspace_bytes(0, 256, 1024) == 0


def _fused(lib, prologue=1, src=1 << 16, gamma=1 << 20, rows=16, cols=256, out=1 << 12, odt=0, flags=0,
           bias=None):
    return lib.w4a16_gemv_fused(ctypes.c_void_p(1 << 12), ctypes.c_void_p(1 << 12), 0, 0, prologue,
                                ctypes.c_void_p(src), ctypes.c_void_p(gamma), 1e-5, rows, cols,
                                ctypes.c_void_p(out), odt, bias, None, 0, flags, None)


def test_fused_gemv_host_validation(lib):
    assert _fused(lib, prologue=3) == -4                 # NONE, RMSNorm or SwiGLU only
    assert _fused(lib, prologue=7) == -4
    assert _fused(lib, flags=4) == -4                    # W4A16_LAUNCH_PDL | W4A16_LAUNCH_SWIGLU_OUT only
    # SwiGLU epilogue: RMSNorm prologue, rows in whole 16-row gate / up blocks, no bias
    assert _fused(lib, prologue=0, flags=2) == -2
    assert _fused(lib, prologue=2, flags=2) == -2
    assert _fused(lib, rows=24, flags=2) == -2
    assert _fused(lib, flags=2, bias=ctypes.c_void_p(1 << 24)) == -2
    assert _fused(lib, prologue=0, out=(1 << 16) + 256) == -2   # x fp16 [256] = 512 bytes
    assert _fused(lib, src=0) == -1
    assert _fused(lib, gamma=0) == -1                    # RMSNorm needs gamma
    assert _fused(lib, gamma=(1 << 20) + 4) == -3
    assert _fused(lib, out=(1 << 16) + 512) == -2        # out inside src (fp32 [256] = 1 KiB)
    assert b"overlaps" in lib.w4a16_last_error_string()
    assert _fused(lib, out=(1 << 16) - 32) == -2         # out [16] fp32 runs into src
    assert _fused(lib, cols=200) == -2
    assert _fused(lib, rows=0) == 0                      # empty: no-op before any CUDA call


def _attn(lib, qkv=1 << 12, pos=1 << 13, scratch=1 << 14, scratch_bytes=1 << 20, heads=32,
          kv_heads=8, head_dim=64, max_len=512, splits=16, flags=0):
    p = ctypes.c_void_p
    return lib.w4a16_decode_attention(p(qkv), p(1 << 15), p(1 << 15), p(pos), p(1 << 16), p(1 << 17),
                                      p(1 << 18), p(scratch), scratch_bytes, heads, kv_heads, head_dim,
                                      max_len, splits, flags, None)


def test_decode_attention_host_validation(lib):
    assert lib.w4a16_decode_attention_scratch_bytes(32, 8, 16) == (32 * 16 * 66 + 8) * 4
    assert lib.w4a16_decode_attention_scratch_bytes(0, 8, 16) == 0
    assert _attn(lib, qkv=0) == -1
    assert _attn(lib, head_dim=128) == -2
    assert _attn(lib, kv_heads=5) == -2                  # heads % kv_heads
    assert _attn(lib, heads=64, kv_heads=1) == -2        # more than 32 query heads per kv head
    assert _attn(lib, splits=0) == -2
    assert _attn(lib, splits=600) == -2                  # more splits than positions
    assert _attn(lib, max_len=0) == -2
    assert _attn(lib, qkv=(1 << 12) + 2) == -3
    assert _attn(lib, pos=(1 << 13) + 4) == -3
    assert _attn(lib, scratch_bytes=100) == -5
    assert b"scratch" in lib.w4a16_last_error_string()
    assert _attn(lib, flags=4) == -4


def test_tensor_parallel_host_validation(lib):
    assert lib.w4a16_tp_header_bytes() == 256
    assert lib.w4a16_tp_ipc_handle_bytes() == 64
    p = ctypes.c_void_p
    assert lib.w4a16_tp_region_alloc(1024, None, None) == -1
    assert lib.w4a16_tp_region_open(None, None) == -1
    assert lib.w4a16_tp_region_close(None, 1) == 0

    def call(regions=((1 << 20), (2 << 20)), rank=0, nranks=2, rows=16, row0=0, cols=256, flags=0):
        arr = (ctypes.c_void_p * len(regions))(*regions) if regions is not None else None
        return lib.w4a16_gemv_allgather(p(1 << 12), p(1 << 12), 0, 0, p(1 << 16), rows, cols, 0, row0,
                                        rank, nranks, arr, None, 0, flags, None)

    assert call(regions=None) == -1
    assert call(nranks=1) == -2
    assert call(nranks=9) == -2
    assert call(rank=2) == -2
    assert call(rows=0) == -2
    assert call(row0=-16) == -2
    assert call(regions=((1 << 20), (2 << 20) + 64)) == -3   # regions 256-byte aligned
    assert call(regions=((1 << 20), 0)) == -1
    assert call(cols=200) == -2
    assert call(flags=2) == -4
    # regions the process neither allocated nor opened: their capacity is unknown
    assert call() == -2
    assert b"w4a16_tp_region_alloc" in lib.w4a16_last_error_string()
    assert lib.w4a16_tp_set_peer_wait_ns(999) == -2
    assert lib.w4a16_tp_set_peer_wait_ns(61 * 10**9) == -2
    assert lib.w4a16_tp_set_peer_wait_ns(50 * 10**6) == 0
    assert lib.w4a16_tp_set_peer_wait_ns(0) == 0


def test_decode_plan_host_validation(lib):
    """The one-kernel decode step checks its model description on the host before any
    CUDA call (no GPU needed for these answers)."""
    from w4a16.decode import _G128Weight, _LlamaDesc

    plan = ctypes.c_void_p()
    assert lib.w4a16_decode_plan_create(None, ctypes.byref(plan)) == -1
    assert lib.w4a16_decode_plan_create(None, None) == -1
    w = (_G128Weight * 1)(_G128Weight(1 << 12, 1 << 12))
    n = (ctypes.c_void_p * 1)(1 << 12)

    def desc(**kw):
        f = dict(layers=1, hidden=2048, intermediate=8192, heads=32, kv_heads=8, head_dim=64, vocab=1000,
                 max_len=64, eps=1e-5)
        f.update(kw)
        return _LlamaDesc(f["layers"], f["hidden"], f["intermediate"], f["heads"], f["kv_heads"], f["head_dim"],
                          f["vocab"], f["max_len"], f["eps"], w, w, w, w, n, n, _G128Weight(1 << 12, 1 << 12),
                          1 << 12, 1 << 12, 1 << 12, 1 << 12)

    for bad in (dict(head_dim=128), dict(hidden=2000), dict(heads=30), dict(heads=64, kv_heads=4),
                dict(layers=0), dict(intermediate=32768), dict(max_len=0), dict(hidden=8192),
                dict(intermediate=2560), dict(intermediate=9216), dict(heads=72, kv_heads=9)):
        assert lib.w4a16_decode_plan_create(ctypes.byref(desc(**bad)), ctypes.byref(plan)) == -2, bad
    assert b"unsupported decode-step shape" in lib.w4a16_last_error_string()
    p = ctypes.c_void_p
    assert lib.w4a16_decode_step(None, p(8), p(8), p(16), p(16), p(4), None) == -1
    assert lib.w4a16_decode_step(p(1 << 12), p(8), p(12), p(16), p(16), p(4), None) == -3
    assert lib.w4a16_decode_plan_destroy(None) == 0
