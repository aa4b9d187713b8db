// w4a16_gemv_noalloc: the split-K W4A16 GEMV for callers that cannot allocate.
//
// Some callers hand this library only their input and output buffers and cannot
// give it any other device memory: a runtime that plans all device memory at
// start-up and forbids allocation afterwards (cudaMalloc may synchronise the whole
// device and breaks such a plan), or a plugin interface whose op signature has no
// workspace argument.  The GEMV still needs scratch memory to balance its work
// across warps (per-warp counters plus fp32 partial sums of the tiles that
// neighbouring warps share; about 0.5 MiB for one activation vector, whatever the
// matrix size).  This entry point takes that scratch from a fixed array that lives
// in the library itself, so it calls no cudaMalloc, cudaFree or allocating routine.
//
// The array (kNoAllocScratchBytes, 4 MiB) is a file-scope __device__ variable: every
// GPU that loads the library holds one copy until the process exits.  Every call on
// a device shares that one copy and leaves its contents behind; the counters that
// must start at zero are cleared on the caller's stream at the start of each call.
// Calls whose executions overlap on the GPU (different streams without ordering
// between them) race on the array and give wrong results: order them on one stream.
//
// Host code never uses the array's name as a device address (on the host it names a
// stand-in object).  The first call on each device, with that device current, asks
// the runtime for the array's device address with cudaGetSymbolAddress and caches
// it; make that first call before any stream capture on the device.  The cache is
// keyed by the device and by its current CUDA context, so a caller that switches to
// another context, or whose context was destroyed (cudaDeviceReset) and recreated,
// gets the address looked up again in the new context.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "w4a16_b200.h"
#include "w4a16_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)4 << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// cuCtxGetCurrent from the driver the runtime already loaded (no link against libcuda).
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  });
  return fn;
}

// Device address of the scratch array on the current device, looked up once per
// (device, context) and cached.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    w4a16::set_error("cudaGetDevice: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    w4a16::set_error("device index %d out of range", dev);
    return W4A16_ERR_CUDA;
  }
  CtxGetCurrentFn get_ctx = ctx_get_current();
  if (!get_ctx) {
    w4a16::set_error("cuCtxGetCurrent is unavailable");
    return W4A16_ERR_CUDA;
  }
  CUcontext ctx = nullptr;  // null while no context is current on this thread
  if (get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!ctx || !g_scratch_addr[dev] || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    // (makes the device's primary context current when none is)
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      w4a16::set_error("cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
      return W4A16_ERR_CUDA;
    }
    if (get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    g_scratch_addr[dev] = p;
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_addr[dev];
  return W4A16_OK;
}

}  // namespace

extern "C" int w4a16_gemv_noalloc(const uint8_t* packed, const void* scale, int scale_dtype,
                                  int group, const void* x, int rows, int cols, float* out,
                                  w4a16_stream_t stream) {
  if (rows < 0 || cols <= 0 || cols % 8 != 0) {
    w4a16::set_error("bad shape rows=%d cols=%d", rows, cols);
    return W4A16_ERR_SHAPE;
  }
  if ((scale_dtype != W4A16_DTYPE_F32 && scale_dtype != W4A16_DTYPE_F16) ||
      (group != 0 && group != 128)) {
    w4a16::set_error("bad scale dtype %d or group %d", scale_dtype, group);
    return W4A16_ERR_DTYPE;
  }
  if (group && cols % group != 0) {
    w4a16::set_error("cols=%d must be a multiple of %d", cols, group);
    return W4A16_ERR_SHAPE;
  }
  if (rows == 0) return W4A16_OK;
  if (!packed || !scale || !x || !out) {
    w4a16::set_error("NULL pointer");
    return W4A16_ERR_NULL;
  }
  const size_t need = w4a16::gemv_workspace_bytes(1, rows, cols);
  if (need > kNoAllocScratchBytes) {
    w4a16::set_error(
        "w4a16_gemv_noalloc: rows=%d cols=%d needs %zu bytes of scratch, more than the %zu-byte "
        "static array; use w4a16_gemv with a workspace",
        rows, cols, need, kNoAllocScratchBytes);
    return W4A16_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != W4A16_OK) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const cudaError_t e = cudaMemsetAsync(scratch, 0, w4a16::gemv_counter_bytes(), s);
  if (e != cudaSuccess) {
    w4a16::set_error("clearing the scratch counters: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  return w4a16_gemv(packed, W4A16_PACK_INTERLEAVED, scale, scale_dtype, group, x, 1, rows, cols,
                    out, W4A16_DTYPE_F32, nullptr, scratch, kNoAllocScratchBytes, stream);
}
