"""Ahead-of-time build of libw4a16_b200.so (the C-ABI CUDA library) for sm_100a.

The reference JIT-compiles its kernels with torch.utils.cpp_extension.load() on
first use (src/w4a16/kernels.py:24-29).  Here the library is a plain shared object
with an extern "C" interface, compiled by nvcc once, in-tree, so it ships with the
package and loads without a compiler:

    python -m w4a16.build            # from the package root directory
"""
import concurrent.futures
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)                      # w4a16-gemv-optimization-ladder_b200/
CSRC_DIR = os.path.join(ROOT_DIR, "csrc")
INCLUDE_DIR = os.path.join(os.path.dirname(ROOT_DIR), "include")
BUILD_DIR = os.path.join(ROOT_DIR, "_build")
LIB_NAME = "libw4a16_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

SOURCES = ["w4a16_gemv.cu", "w4a16_aux.cu", "w4a16_capi.cu", "w4a16_noalloc.cu", "w4a16_decode.cu",
           "w4a16_decode_step.cu", "w4a16_gemm.cu"]
HEADERS = ["w4a16_device.cuh", "w4a16_gemv_core.cuh", "w4a16_internal.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
]


def _nvcc():
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libw4a16_b200.so")
    return cand


def _newest(paths):
    return max(os.path.getmtime(p) for p in paths)


def _compile(nvcc, src, obj, defines, verbose):
    cmd = [nvcc, *NVCC_FLAGS, *[f"-D{d}" for d in defines], "-I", INCLUDE_DIR, "-I", CSRC_DIR,
           "-c", os.path.join(CSRC_DIR, src), "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    return res.stderr


def build(force=False, verbose=False, defines=(), out=None):
    """Compile every CUDA source for sm_100a and link the shared library.

    Rebuilds only when a source or header is newer than the library (or `force`).
    Returns the path of the library.
    """
    out = out or LIB_PATH
    srcs = [os.path.join(CSRC_DIR, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC_DIR, h) for h in HEADERS] + [
        os.path.join(INCLUDE_DIR, "w4a16_b200.h"), os.path.abspath(__file__)]
    if not force and not defines and os.path.exists(out) and os.path.getmtime(out) >= _newest(deps):
        return out
    nvcc = _nvcc()
    tag = "_".join(d.replace("=", "") for d in defines) or "default"
    bdir = os.path.join(BUILD_DIR, tag)
    os.makedirs(bdir, exist_ok=True)
    objs = [os.path.join(bdir, s.replace(".cu", ".o")) for s in SOURCES]
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        logs = list(ex.map(lambda so: _compile(nvcc, so[0], so[1], defines, verbose),
                           zip(SOURCES, objs)))
    if verbose:
        for s, log in zip(SOURCES, logs):
            print(f"--- {s}\n{log}")
    tmp = out + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-lcudart_static", "-ldl", "-lrt",
           "-lpthread"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    v = "-v" in sys.argv
    print(build(force="--force" in sys.argv, verbose=v))
