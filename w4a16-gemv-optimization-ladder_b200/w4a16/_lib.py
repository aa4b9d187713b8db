"""ctypes binding of libw4a16_b200.so, the C-ABI CUDA library (include/w4a16_b200.h).

This is the boundary the reference crossed with a pybind11 module JIT-built by
torch.utils.cpp_extension.load (src/w4a16/kernels.py:24-29): here the kernels sit
behind plain extern "C" functions taking device pointers, sizes and a stream.
There is no fallback: if the library is missing every op raises.
"""
import ctypes
import functools
import os

LIB_NAME = "libw4a16_b200.so"
ENV_LIB = "W4A16_B200_LIB"

W4A16_OK = 0
DTYPE_F32 = 0
DTYPE_F16 = 1
PACK_INTERLEAVED = 0
PACK_SIMPLE = 1
PROLOGUE_NONE = 0
PROLOGUE_RMSNORM = 1
PROLOGUE_SWIGLU = 2
LAUNCH_PDL = 1
LAUNCH_SWIGLU_OUT = 2

_p = ctypes.c_void_p
_i = ctypes.c_int
_u = ctypes.c_uint
_sz = ctypes.c_size_t

_REF_SIG = [_p, _p, _p, _p, _i, _i, _p]
SIGNATURES = {
    # name: (argtypes, restype)
    "w4a16_marlin_cuda": (_REF_SIG, _i),
    "w4a16_marlin_g128_cuda": (_REF_SIG, _i),
    "w4a16_byte_cuda": (_REF_SIG, _i),
    "w4a16_u32_cuda": (_REF_SIG, _i),
    "w4a16_u32_v4_cuda": (_REF_SIG, _i),
    "w4a16_champ_cuda": (_REF_SIG, _i),
    "w4a16_uint4_cuda": (_REF_SIG, _i),
    "w4a16_h2f32_cuda": (_REF_SIG, _i),
    "w4a16_fp16_cuda": ([_p, _p, _p, _i, _i, _p], _i),
    "w4a16_gemv": ([_p, _i, _p, _i, _i, _p, _i, _i, _i, _p, _i, _p, _p, _sz, _p], _i),
    "w4a16_gemv_workspace_bytes": ([_i, _i, _i], _sz),
    "w4a16_gemv_fused": ([_p, _p, _i, _i, _i, _p, _p, ctypes.c_float, _i, _i, _p, _i, _p, _p, _sz, _u, _p],
                         _i),
    "w4a16_decode_attention": ([_p, _p, _p, _p, _p, _p, _p, _p, _sz, _i, _i, _i, _i, _i, _u, _p], _i),
    "w4a16_decode_attention_scratch_bytes": ([_i, _i, _i], _sz),
    "w4a16_tp_header_bytes": ([], _sz),
    "w4a16_tp_ipc_handle_bytes": ([], _sz),
    "w4a16_tp_region_alloc": ([_sz, ctypes.POINTER(ctypes.c_void_p), _p], _i),
    "w4a16_tp_region_open": ([_p, ctypes.POINTER(ctypes.c_void_p)], _i),
    "w4a16_tp_region_close": ([_p, _i], _i),
    "w4a16_gemv_allgather": ([_p, _p, _i, _i, _p, _i, _i, _i, ctypes.c_longlong, _i, _i,
                              ctypes.POINTER(ctypes.c_void_p), _p, _sz, _u, _p], _i),
    "w4a16_tp_set_peer_wait_ns": ([ctypes.c_ulonglong], _i),
    "w4a16_tp_region_timeline": ([_p, _p, _p], _i),
    "w4a16_decode_plan_create": ([_p, ctypes.POINTER(ctypes.c_void_p)], _i),
    "w4a16_decode_plan_destroy": ([_p], _i),
    "w4a16_decode_step": ([_p, _p, _p, _p, _p, _p, _p], _i),
    "w4a16_decode_plan_timeline": ([_p, _i, _p, _sz, ctypes.POINTER(_sz), _p], _i),
    "w4a16_gemv_noalloc": ([_p, _p, _i, _i, _p, _i, _i, _p, _p], _i),
    "w4a16_dequant": ([_p, _i, _p, _i, _i, _i, _i, _p, _p], _i),
    "w4a16_quantize_pack": ([_p, _i, _i, _i, _i, _i, _p, _p, _i, _p], _i),
    "w4a16_gemm": ([_p, _p, _i, _p, _p, _i, _i, _i, _p, _i, _p, ctypes.c_size_t, _p], _i),
    "w4a16_gemm_workspace_bytes": ([_i, _i, _i], ctypes.c_size_t),
    "w4a16_read_device_error": ([ctypes.POINTER(ctypes.c_int), _p], _i),
    "w4a16_status_string": ([_i], ctypes.c_char_p),
    "w4a16_last_error_string": ([], ctypes.c_char_p),
    "w4a16_version": ([], _i),
}


def lib_path():
    """Location of the shared library: $W4A16_B200_LIB, else next to this package."""
    return os.environ.get(ENV_LIB) or os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                   LIB_NAME)


@functools.lru_cache(maxsize=1)
def lib():
    """Load the library once and attach the C signatures; raise if it is missing."""
    path = lib_path()
    if not os.path.exists(path):
        raise RuntimeError(
            f"w4a16 CUDA library not found at {path}: build it with `python -m w4a16.build` "
            "(there is no CPU fallback)")
    handle = ctypes.CDLL(path)
    for name, (argtypes, restype) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.argtypes = argtypes
        fn.restype = restype
    return handle


def check(status, what):
    """Raise RuntimeError carrying the library's message for a non-zero status."""
    if status != W4A16_OK:
        L = lib()
        msg = L.w4a16_last_error_string().decode(errors="replace")
        raise RuntimeError(f"{what}: {L.w4a16_status_string(status).decode()} ({msg})")
