"""TEST INFRASTRUCTURE ONLY — ctypes access to the C oracle (oracle/w4a16_oracle.c).

Same algorithm as oracle/w4a16_oracle.py, in C with OpenMP, for full-size checks and
for the timed CPU baseline.  Built by `make -C oracle` (or __graft_entry__.build()).
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle_w4a16.so")


def build():
    """Compile the C oracle if the shared object is missing or stale."""
    src = os.path.join(HERE, "w4a16_oracle.c")
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


_handle = None


def lib():
    global _handle
    if _handle is None:
        if not os.path.exists(LIB):
            build()
        h = ctypes.CDLL(LIB)
        p, i = ctypes.c_void_p, ctypes.c_int
        h.oracle_gemv.argtypes = [p, i, p, i, p, i, i, i, p, i, i]
        h.oracle_gemv.restype = i
        h.oracle_quantize_pack.argtypes = [p, i, i, i, i, p, p, i]
        h.oracle_quantize_pack.restype = i
        h.oracle_max_threads.restype = i
        _handle = h
    return _handle


def _ptr(a):
    return ctypes.c_void_p(a.ctypes.data)


def gemv(packed, scale, x, group=0, interleaved=True, accumulate_f64=True, threads=0):
    """y [rows] (x 1-D) or [batch, rows] (x 2-D), fp32, from packed uint8 weights."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float16)
    n, k = packed.shape[0], packed.shape[1] * 2
    m = 1 if x.ndim == 1 else x.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    rc = lib().oracle_gemv(_ptr(packed), int(interleaved), _ptr(scale), group, _ptr(x.view(np.uint16)),
                           m, n, k, _ptr(y), int(accumulate_f64), threads)
    if rc != 0:
        raise RuntimeError(f"oracle_gemv failed ({rc})")
    return y[0] if x.ndim == 1 else y


def quantize_pack(w, group=0, interleaved=True, threads=0):
    """(packed uint8 [rows, cols/2], scale fp32 [rows] or [rows, cols/group])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    packed = np.empty((rows, cols // 2), dtype=np.uint8)
    scale = np.empty((rows,) if group == 0 else (rows, cols // group), dtype=np.float32)
    rc = lib().oracle_quantize_pack(_ptr(w), rows, cols, group, int(interleaved), _ptr(packed),
                                    _ptr(scale), threads)
    if rc != 0:
        raise RuntimeError(f"oracle_quantize_pack failed ({rc})")
    return packed, scale


def max_threads():
    return int(lib().oracle_max_threads())
