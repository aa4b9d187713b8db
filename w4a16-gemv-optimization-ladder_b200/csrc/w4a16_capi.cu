// extern "C" entry points of libw4a16_b200.so (declared in include/w4a16_b200.h).
// Host-side validation happens here, before anything is launched: a bad pointer,
// shape, alignment or dtype code returns a status and launches nothing.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <unordered_map>

#include "w4a16_b200.h"
#include "w4a16_internal.h"

namespace {

using w4a16::set_error;

constexpr int kVersion = 1 * 10000 + 0 * 100 + 0;

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Tensor-parallel regions known to this process (created by w4a16_tp_region_alloc or
// mapped by w4a16_tp_region_open), with the byte capacity of each one's gathered output.
// The fused all-gather stores every rank's rows into every region, so a call whose rows
// do not fit one of them is rejected before launch.  The capacity also sits in the
// region's header (kTpCapacityOffset), where the opening process reads it.
std::mutex g_region_mu;
std::unordered_map<uintptr_t, size_t> g_region_capacity;

void register_region(void* region, size_t out_bytes) {
  std::lock_guard<std::mutex> lock(g_region_mu);
  g_region_capacity[reinterpret_cast<uintptr_t>(region)] = out_bytes;
}

void forget_region(void* region) {
  std::lock_guard<std::mutex> lock(g_region_mu);
  g_region_capacity.erase(reinterpret_cast<uintptr_t>(region));
}

bool region_capacity(const void* region, size_t* out_bytes) {
  std::lock_guard<std::mutex> lock(g_region_mu);
  const auto it = g_region_capacity.find(reinterpret_cast<uintptr_t>(region));
  if (it == g_region_capacity.end()) return false;
  *out_bytes = it->second;
  return true;
}

// Limit of the fused all-gather's waits on other GPUs (0 = the 2 s default).
std::atomic<unsigned long long> g_peer_wait_ns{0};
constexpr unsigned long long kDefaultPeerWaitNs = 2000000000ull;

// Shape / pointer checks shared by every GEMV-style entry point.
int check_gemv(const void* packed, int packing, const void* scale, int scale_dtype, int group,
               const void* x, int batch, int rows, int cols, const void* out, int out_dtype) {
  if (packing != W4A16_PACK_INTERLEAVED && packing != W4A16_PACK_SIMPLE) {
    set_error("unknown packing code %d", packing);
    return W4A16_ERR_DTYPE;
  }
  if ((scale_dtype != W4A16_DTYPE_F32 && scale_dtype != W4A16_DTYPE_F16) ||
      (out_dtype != W4A16_DTYPE_F32 && out_dtype != W4A16_DTYPE_F16)) {
    set_error("unknown dtype code (scale %d, out %d)", scale_dtype, out_dtype);
    return W4A16_ERR_DTYPE;
  }
  if (group != 0 && group != 128) {
    set_error("group must be 0 (per-row) or 128, got %d", group);
    return W4A16_ERR_DTYPE;
  }
  if (rows < 0 || cols <= 0 || batch < 0) {
    set_error("bad shape rows=%d cols=%d batch=%d", rows, cols, batch);
    return W4A16_ERR_SHAPE;
  }
  if (cols % 8 != 0 || (group && cols % group != 0)) {
    set_error("cols=%d must be a multiple of %d", cols, group ? group : 8);
    return W4A16_ERR_SHAPE;
  }
  if (rows == 0 || batch == 0) return W4A16_OK;
  if (!packed || !scale || !x || !out) {
    set_error("NULL pointer (packed %p, scale %p, x %p, out %p)", packed, scale, x, out);
    return W4A16_ERR_NULL;
  }
  const size_t ssz = scale_dtype == W4A16_DTYPE_F32 ? 4 : 2;
  const size_t osz = out_dtype == W4A16_DTYPE_F32 ? 4 : 2;
  if (!aligned(packed, 4) || !aligned(x, 16) || !aligned(scale, ssz) || !aligned(out, osz)) {
    set_error("misaligned pointer: packed needs 4 B, x 16 B, scale %zu B, out %zu B", ssz, osz);
    return W4A16_ERR_ALIGN;
  }
  return W4A16_OK;
}

int gemv_common(const uint8_t* packed, int packing, const void* scale, int scale_dtype, int group,
                const void* x, int batch, int rows, int cols, void* out, int out_dtype,
                const float* bias, void* workspace, size_t workspace_bytes,
                w4a16_stream_t stream) {
  int rc = check_gemv(packed, packing, scale, scale_dtype, group, x, batch, rows, cols, out,
                      out_dtype);
  if (rc != W4A16_OK || rows == 0 || batch == 0) return rc;
  if (bias && !aligned(bias, 4)) {
    set_error("bias must be 4-byte aligned");
    return W4A16_ERR_ALIGN;
  }
  w4a16::GemvProblem p;
  p.packed = packed;
  p.packing = packing;
  p.scale = scale;
  p.scale_dtype = scale_dtype;
  p.group = group;
  p.x = x;
  p.M = batch;
  p.N = rows;
  p.K = cols;
  p.y = out;
  p.out_dtype = out_dtype;
  p.bias = bias;
  p.workspace = workspace;
  p.workspace_bytes = workspace ? workspace_bytes : 0;
  p.split_k = 0;
  p.stream = reinterpret_cast<cudaStream_t>(stream);
  return w4a16::launch_gemv(p);
}

int ladder(const uint8_t* packed, const float* scale, const void* vec, float* out, int rows,
           int cols, w4a16_stream_t stream) {
  return gemv_common(packed, W4A16_PACK_SIMPLE, scale, W4A16_DTYPE_F32, 0, vec, 1, rows, cols, out,
                     W4A16_DTYPE_F32, nullptr, nullptr, 0, stream);
}

}  // namespace

extern "C" {

int w4a16_marlin_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                      int rows, int cols, w4a16_stream_t stream) {
  return gemv_common(packed, W4A16_PACK_INTERLEAVED, scale, W4A16_DTYPE_F32, 0, vec, 1, rows, cols,
                     out, W4A16_DTYPE_F32, nullptr, nullptr, 0, stream);
}

int w4a16_marlin_g128_cuda(const uint8_t* packed, const float* scale, const void* vec,
                           float* out, int rows, int cols, w4a16_stream_t stream) {
  return gemv_common(packed, W4A16_PACK_INTERLEAVED, scale, W4A16_DTYPE_F32, 128, vec, 1, rows,
                     cols, out, W4A16_DTYPE_F32, nullptr, nullptr, 0, stream);
}

int w4a16_byte_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                    int rows, int cols, w4a16_stream_t stream) {
  return ladder(packed, scale, vec, out, rows, cols, stream);
}

int w4a16_u32_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                   int rows, int cols, w4a16_stream_t stream) {
  return ladder(packed, scale, vec, out, rows, cols, stream);
}

int w4a16_u32_v4_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                      int rows, int cols, w4a16_stream_t stream) {
  return ladder(packed, scale, vec, out, rows, cols, stream);
}

int w4a16_champ_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                     int rows, int cols, w4a16_stream_t stream) {
  return ladder(packed, scale, vec, out, rows, cols, stream);
}

int w4a16_uint4_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                     int rows, int cols, w4a16_stream_t stream) {
  return ladder(packed, scale, vec, out, rows, cols, stream);
}

int w4a16_h2f32_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                     int rows, int cols, w4a16_stream_t stream) {
  int rc = check_gemv(packed, W4A16_PACK_SIMPLE, scale, W4A16_DTYPE_F32, 0, vec, 1, rows, cols,
                      out, W4A16_DTYPE_F32);
  if (rc != W4A16_OK || rows == 0) return rc;
  return w4a16::launch_h2f32(packed, scale, vec, out, rows, cols,
                             reinterpret_cast<cudaStream_t>(stream));
}

int w4a16_fp16_cuda(const void* mat, const void* vec, float* out, int rows, int cols,
                    w4a16_stream_t stream) {
  if (rows < 0 || cols <= 0 || cols % 8 != 0) {
    set_error("bad shape rows=%d cols=%d (cols must be a positive multiple of 8)", rows, cols);
    return W4A16_ERR_SHAPE;
  }
  if (rows == 0) return W4A16_OK;
  if (!mat || !vec || !out) {
    set_error("NULL pointer");
    return W4A16_ERR_NULL;
  }
  if (!aligned(mat, 16) || !aligned(vec, 16) || !aligned(out, 4)) {
    set_error("mat and vec must be 16-byte aligned, out 4-byte aligned");
    return W4A16_ERR_ALIGN;
  }
  return w4a16::launch_fp16_gemv(mat, vec, out, rows, cols, reinterpret_cast<cudaStream_t>(stream));
}

int w4a16_gemv(const uint8_t* packed, int packing, const void* scale, int scale_dtype, int group,
               const void* x, int batch, int rows, int cols, void* out, int out_dtype,
               const float* bias, void* workspace, size_t workspace_bytes,
               w4a16_stream_t stream) {
  return gemv_common(packed, packing, scale, scale_dtype, group, x, batch, rows, cols, out,
                     out_dtype, bias, workspace, workspace_bytes, stream);
}

int w4a16_gemv_fused(const uint8_t* packed, const void* scale, int scale_dtype, int group,
                     int prologue, const void* src, const float* gamma, float eps, int rows,
                     int cols, void* out, int out_dtype, const float* bias, void* workspace,
                     size_t workspace_bytes, unsigned flags, w4a16_stream_t stream) {
  if (prologue != W4A16_PROLOGUE_NONE && prologue != W4A16_PROLOGUE_RMSNORM &&
      prologue != W4A16_PROLOGUE_SWIGLU) {
    set_error("unknown prologue code %d", prologue);
    return W4A16_ERR_DTYPE;
  }
  if (flags & ~(unsigned)(W4A16_LAUNCH_PDL | W4A16_LAUNCH_SWIGLU_OUT)) {
    set_error("unknown launch flags 0x%x", flags);
    return W4A16_ERR_DTYPE;
  }
  const bool swiglu_out = (flags & W4A16_LAUNCH_SWIGLU_OUT) != 0;
  if (swiglu_out && (prologue != W4A16_PROLOGUE_RMSNORM || bias || rows % 16 != 0)) {
    set_error("W4A16_LAUNCH_SWIGLU_OUT needs the RMSNorm prologue, no bias and rows %% 16 == 0 (got %d)",
              rows);
    return W4A16_ERR_SHAPE;
  }
  // src stands in for x in the shared checks (16-byte alignment, non-NULL)
  int rc = check_gemv(packed, W4A16_PACK_INTERLEAVED, scale, scale_dtype, group, src, 1, rows, cols,
                      out, out_dtype);
  if (rc != W4A16_OK || rows == 0) return rc;
  if (cols % 256 != 0 || !aligned(packed, 16)) {
    set_error("fused prologue needs cols %% 256 == 0 (got %d) and 16-byte aligned weights", cols);
    return cols % 256 != 0 ? W4A16_ERR_SHAPE : W4A16_ERR_ALIGN;
  }
  if (prologue == W4A16_PROLOGUE_RMSNORM && (!gamma || !aligned(gamma, 16))) {
    set_error("rmsnorm prologue needs a 16-byte aligned gamma");
    return gamma ? W4A16_ERR_ALIGN : W4A16_ERR_NULL;
  }
  if (bias && !aligned(bias, 4)) {
    set_error("bias must be 4-byte aligned");
    return W4A16_ERR_ALIGN;
  }
  {  // every CTA reads all of src while rows of out are written
    const uintptr_t s0 = reinterpret_cast<uintptr_t>(src);
    const uintptr_t s1 = s0 + (size_t)cols * (prologue == W4A16_PROLOGUE_NONE ? 2 : 4);
    const uintptr_t o0 = reinterpret_cast<uintptr_t>(out);
    const uintptr_t o1 = o0 + (size_t)(swiglu_out ? rows / 2 : rows) * (out_dtype == W4A16_DTYPE_F32 ? 4 : 2);
    if (s0 < o1 && o0 < s1) {
      set_error("out overlaps the prologue source");
      return W4A16_ERR_SHAPE;
    }
  }
  w4a16::GemvProblem p;
  p.packed = packed;
  p.packing = W4A16_PACK_INTERLEAVED;
  p.scale = scale;
  p.scale_dtype = scale_dtype;
  p.group = group;
  p.x = src;
  p.M = 1;
  p.N = rows;
  p.K = cols;
  p.y = out;
  p.out_dtype = out_dtype;
  p.bias = bias;
  p.workspace = workspace;
  p.workspace_bytes = workspace ? workspace_bytes : 0;
  p.prologue = prologue;
  p.pro_src = src;
  p.pro_gamma = gamma;
  p.pro_eps = eps;
  p.staged = true;
  p.pdl = (flags & W4A16_LAUNCH_PDL) != 0;
  p.out_swiglu = swiglu_out;
  p.stream = reinterpret_cast<cudaStream_t>(stream);
  return w4a16::launch_gemv(p);
}

int w4a16_decode_attention(const void* qkv, const float* cos_t, const float* sin_t,
                           const int64_t* pos, void* k_cache, void* v_cache, void* out,
                           void* scratch, size_t scratch_bytes, int heads, int kv_heads,
                           int head_dim, int max_len, int splits, unsigned flags,
                           w4a16_stream_t stream) {
  if (flags & ~(unsigned)W4A16_LAUNCH_PDL) {
    set_error("unknown launch flags 0x%x", flags);
    return W4A16_ERR_DTYPE;
  }
  if (!qkv || !cos_t || !sin_t || !pos || !k_cache || !v_cache || !out || !scratch) {
    set_error("null pointer argument");
    return W4A16_ERR_NULL;
  }
  if (head_dim != 64 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 ||
      heads / kv_heads > 32 || max_len <= 0 || splits <= 0 || splits > max_len) {
    set_error("unsupported attention shape: heads %d kv_heads %d head_dim %d max_len %d splits %d "
              "(head_dim 64, heads %% kv_heads == 0, heads / kv_heads <= 32, 1 <= splits <= max_len)",
              heads, kv_heads, head_dim, max_len, splits);
    return W4A16_ERR_SHAPE;
  }
  if (!aligned(qkv, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(out, 16) ||
      !aligned(cos_t, 4) || !aligned(sin_t, 4) || !aligned(pos, 8) || !aligned(scratch, 4)) {
    set_error("qkv, caches and out must be 16-byte aligned; tables and scratch 4; pos 8");
    return W4A16_ERR_ALIGN;
  }
  if (scratch_bytes < w4a16::decode_attention_scratch_bytes(heads, kv_heads, splits)) {
    set_error("scratch of %zu bytes is smaller than the %zu needed", scratch_bytes,
              w4a16::decode_attention_scratch_bytes(heads, kv_heads, splits));
    return W4A16_ERR_WORKSPACE;
  }
  return w4a16::launch_decode_attention(qkv, cos_t, sin_t, reinterpret_cast<const long long*>(pos),
                                        k_cache, v_cache, out, scratch, heads, kv_heads, head_dim,
                                        max_len, splits, (flags & W4A16_LAUNCH_PDL) != 0,
                                        reinterpret_cast<cudaStream_t>(stream));
}

size_t w4a16_decode_attention_scratch_bytes(int heads, int kv_heads, int splits) {
  if (heads <= 0 || kv_heads <= 0 || splits <= 0) return 0;
  return w4a16::decode_attention_scratch_bytes(heads, kv_heads, splits);
}

size_t w4a16_tp_header_bytes(void) { return w4a16::kTpHeaderBytes; }

size_t w4a16_tp_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int w4a16_tp_region_alloc(size_t out_bytes, void** region, void* ipc_handle) {
  if (!region || !ipc_handle) {
    set_error("null pointer argument");
    return W4A16_ERR_NULL;
  }
  *region = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, w4a16::kTpHeaderBytes + out_bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, w4a16::kTpHeaderBytes + out_bytes);
  if (e == cudaSuccess) {  // the output capacity, for the processes that open the region
    const unsigned long long cap = out_bytes;
    e = cudaMemcpy(static_cast<uint8_t*>(p) + w4a16::kTpCapacityOffset, &cap, sizeof(cap),
                   cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    set_error("tensor-parallel region of %zu bytes: %s", out_bytes, cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  register_region(p, out_bytes);
  *region = p;
  return W4A16_OK;
}

int w4a16_tp_region_open(const void* ipc_handle, void** region) {
  if (!region || !ipc_handle) {
    set_error("null pointer argument");
    return W4A16_ERR_NULL;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  unsigned long long cap = 0;  // written into the header by the owner's w4a16_tp_region_alloc
  e = cudaMemcpy(&cap, static_cast<uint8_t*>(p) + w4a16::kTpCapacityOffset, sizeof(cap),
                 cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    cudaIpcCloseMemHandle(p);
    set_error("reading the capacity of an opened region: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  register_region(p, (size_t)cap);
  *region = p;
  return W4A16_OK;
}

int w4a16_tp_region_close(void* region, int owned) {
  if (!region) return W4A16_OK;
  forget_region(region);
  const cudaError_t e = owned ? cudaFree(region) : cudaIpcCloseMemHandle(region);
  if (e != cudaSuccess) {
    set_error("closing a tensor-parallel region: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  return W4A16_OK;
}

int w4a16_tp_region_timeline(const void* region, unsigned long long* stamps, w4a16_stream_t stream) {
  if (!region || !stamps) {
    set_error("null pointer argument");
    return W4A16_ERR_NULL;
  }
  size_t cap = 0;
  if (!region_capacity(region, &cap)) {
    set_error("region %p was not created by w4a16_tp_region_alloc or mapped by w4a16_tp_region_open in this process", region);
    return W4A16_ERR_SHAPE;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(stamps, static_cast<const uint8_t*>(region) + w4a16::kTpTimelineOffset,
                                  4 * sizeof(unsigned long long), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    set_error("reading a region's step timeline: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  return W4A16_OK;
}

int w4a16_gemv_allgather(const uint8_t* packed, const void* scale, int scale_dtype, int group,
                         const void* x, int rows, int cols, int out_dtype, long long row0, int rank,
                         int nranks, void* const* regions, void* workspace, size_t workspace_bytes,
                         unsigned flags, w4a16_stream_t stream) {
  if (flags & ~(unsigned)W4A16_LAUNCH_PDL) {
    set_error("unknown launch flags 0x%x", flags);
    return W4A16_ERR_DTYPE;
  }
  if (!regions) {
    set_error("null pointer argument");
    return W4A16_ERR_NULL;
  }
  if (nranks < 2 || nranks > 8 || rank < 0 || rank >= nranks || row0 < 0 || rows < 1) {
    set_error("fused all-gather needs 2..8 ranks, 0 <= rank < nranks, row0 >= 0 and rows >= 1 "
              "(got rank %d of %d, row0 %lld, rows %d)", rank, nranks, row0, rows);
    return W4A16_ERR_SHAPE;
  }
  for (int k = 0; k < nranks; ++k)
    if (!regions[k] || !aligned(regions[k], 256)) {
      set_error("region %d is null or not 256-byte aligned", k);
      return regions[k] ? W4A16_ERR_ALIGN : W4A16_ERR_NULL;
    }
  uint8_t* mine = static_cast<uint8_t*>(regions[rank]) + w4a16::kTpHeaderBytes;
  int rc = check_gemv(packed, W4A16_PACK_INTERLEAVED, scale, scale_dtype, group, x, 1, rows, cols,
                      mine, out_dtype);
  if (rc != W4A16_OK) return rc;
  {  // rows [row0, row0 + rows) are stored into every region: each must hold them
    const size_t esize = out_dtype == W4A16_DTYPE_F32 ? 4 : 2;
    const unsigned long long end = ((unsigned long long)row0 + (unsigned long long)rows) * esize;
    for (int k = 0; k < nranks; ++k) {
      size_t cap = 0;
      if (!region_capacity(regions[k], &cap)) {
        set_error("region %d was not created by w4a16_tp_region_alloc or mapped by "
                  "w4a16_tp_region_open in this process", k);
        return W4A16_ERR_SHAPE;
      }
      if (end > cap) {
        set_error("rows [%lld, %lld) of %zu-byte outputs do not fit region %d (%zu bytes)", row0,
                  row0 + rows, esize, k, cap);
        return W4A16_ERR_SHAPE;
      }
    }
  }
  if (cols % 256 != 0 || !aligned(packed, 16)) {
    set_error("fused all-gather needs cols %% 256 == 0 (got %d) and 16-byte aligned weights", cols);
    return cols % 256 != 0 ? W4A16_ERR_SHAPE : W4A16_ERR_ALIGN;
  }
  w4a16::GemvProblem p;
  p.packed = packed;
  p.packing = W4A16_PACK_INTERLEAVED;
  p.scale = scale;
  p.scale_dtype = scale_dtype;
  p.group = group;
  p.x = x;
  p.M = 1;
  p.N = rows;
  p.K = cols;
  p.y = mine;
  p.out_dtype = out_dtype;
  p.workspace = workspace;
  p.workspace_bytes = workspace ? workspace_bytes : 0;
  p.tp_n = nranks;
  p.tp_rank = rank;
  p.tp_row0 = row0;
  for (int k = 0; k < nranks; ++k) {
    p.tp_flags[k] = static_cast<unsigned*>(regions[k]);
    p.tp_out[k] = static_cast<uint8_t*>(regions[k]) + w4a16::kTpHeaderBytes;
  }
  const unsigned long long wait = g_peer_wait_ns.load(std::memory_order_relaxed);
  p.tp_wait_ns = wait ? wait : kDefaultPeerWaitNs;
  p.pdl = (flags & W4A16_LAUNCH_PDL) != 0;
  p.stream = reinterpret_cast<cudaStream_t>(stream);
  return w4a16::launch_gemv(p);
}

int w4a16_tp_set_peer_wait_ns(unsigned long long ns) {
  if (ns != 0 && (ns < 1000ull || ns > 60000000000ull)) {
    set_error("peer wait limit %llu ns outside [1 us, 60 s] (0 restores the 2 s default)", ns);
    return W4A16_ERR_SHAPE;
  }
  g_peer_wait_ns.store(ns, std::memory_order_relaxed);
  return W4A16_OK;
}

size_t w4a16_gemv_workspace_bytes(int batch, int rows, int cols) {
  return w4a16::gemv_workspace_bytes(batch, rows, cols);
}

int w4a16_dequant(const uint8_t* packed, int packing, const void* scale, int scale_dtype,
                  int group, int rows, int cols, void* out, w4a16_stream_t stream) {
  int rc = check_gemv(packed, packing, scale, scale_dtype, group, out, 1, rows, cols, out,
                      W4A16_DTYPE_F16);
  if (rc != W4A16_OK || rows == 0) return rc;
  return w4a16::launch_dequant(packed, packing, scale, scale_dtype, group, rows, cols, out,
                               reinterpret_cast<cudaStream_t>(stream));
}

int w4a16_quantize_pack(const void* w, int w_dtype, int rows, int cols, int group, int packing,
                        uint8_t* packed, void* scale, int scale_dtype, w4a16_stream_t stream) {
  if (w_dtype != W4A16_DTYPE_F32 && w_dtype != W4A16_DTYPE_F16) {
    set_error("unknown weight dtype code %d", w_dtype);
    return W4A16_ERR_DTYPE;
  }
  int rc = check_gemv(packed, packing, scale, scale_dtype, group, packed, 1, rows, cols, packed,
                      W4A16_DTYPE_F16);
  if (rc != W4A16_OK || rows == 0) return rc;
  if (!w) {
    set_error("NULL weight pointer");
    return W4A16_ERR_NULL;
  }
  if (!aligned(w, w_dtype == W4A16_DTYPE_F32 ? 4 : 2)) {
    set_error("weight pointer misaligned");
    return W4A16_ERR_ALIGN;
  }
  return w4a16::launch_quantize_pack(w, w_dtype, rows, cols, group, packing, packed, scale,
                                     scale_dtype, reinterpret_cast<cudaStream_t>(stream));
}

int w4a16_read_device_error(int* code, w4a16_stream_t stream) {
  if (!code) {
    set_error("NULL code pointer");
    return W4A16_ERR_NULL;
  }
  int a = 0, b = 0, c = 0;
  int rc = w4a16::read_device_error(&a, reinterpret_cast<cudaStream_t>(stream));
  if (rc == W4A16_OK) rc = w4a16::read_decode_step_error(&b, reinterpret_cast<cudaStream_t>(stream));
  if (rc == W4A16_OK) rc = w4a16::read_gemm_error(&c, reinterpret_cast<cudaStream_t>(stream));
  if (rc != W4A16_OK) return rc;
  *code = a ? a : b ? b : c;
  return W4A16_OK;
}

size_t w4a16_gemm_workspace_bytes(int M, int N, int K) { return w4a16::gemm_workspace_bytes(M, N, K); }

int w4a16_gemm(const uint8_t* packed, const float* scale, int group, const void* x,
               const float* bias, int M, int N, int K, void* y, int out_dtype, void* workspace,
               size_t workspace_bytes, w4a16_stream_t stream) {
  if (out_dtype != W4A16_DTYPE_F32 && out_dtype != W4A16_DTYPE_F16) {
    set_error("unknown output dtype code %d", out_dtype);
    return W4A16_ERR_DTYPE;
  }
  if (group != 0 && group != 128) {
    set_error("group must be 0 (per-row) or 128, got %d", group);
    return W4A16_ERR_DTYPE;
  }
  if (M <= 0 || N <= 0 || K <= 0 || K % 64 != 0 || (group && K % group != 0)) {
    set_error("bad GEMM shape M=%d N=%d K=%d (K a multiple of %d)", M, N, K, group ? 128 : 64);
    return W4A16_ERR_SHAPE;
  }
  if (!packed || !scale || !x || !y) {
    set_error("NULL pointer (packed %p, scale %p, x %p, y %p)", (const void*)packed, (const void*)scale,
              x, y);
    return W4A16_ERR_NULL;
  }
  const size_t osz = out_dtype == W4A16_DTYPE_F32 ? 4 : 2;
  if (!aligned(packed, 16) || !aligned(x, 16) || !aligned(scale, 4) || !aligned(y, osz) ||
      (bias && !aligned(bias, 4)) || (workspace && !aligned(workspace, 256))) {
    set_error("misaligned pointer: packed and x need 16 B, scale and bias 4 B, y %zu B, workspace 256 B", osz);
    return W4A16_ERR_ALIGN;
  }
  return w4a16::launch_gemm(packed, scale, group, x, bias, M, N, K, y, out_dtype, workspace,
                            workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int w4a16_decode_plan_create(const w4a16_llama_desc* desc, w4a16_decode_plan* plan) {
  if (!plan) {
    set_error("null plan pointer");
    return W4A16_ERR_NULL;
  }
  w4a16::DecodePlan* p = nullptr;
  const int rc = w4a16::decode_plan_create(desc, &p);
  *plan = reinterpret_cast<w4a16_decode_plan>(p);
  return rc;
}

int w4a16_decode_plan_destroy(w4a16_decode_plan plan) {
  return w4a16::decode_plan_destroy(reinterpret_cast<w4a16::DecodePlan*>(plan));
}

int w4a16_decode_plan_timeline(w4a16_decode_plan plan, int enable, unsigned long long* host,
                               size_t capacity, size_t* count, w4a16_stream_t stream) {
  if (!plan) {
    set_error("null plan");
    return W4A16_ERR_NULL;
  }
  return w4a16::decode_plan_timeline(reinterpret_cast<w4a16::DecodePlan*>(plan), enable, host, capacity,
                                     count, reinterpret_cast<cudaStream_t>(stream));
}

int w4a16_decode_step(w4a16_decode_plan plan, const int64_t* token, const int64_t* pos,
                      void* k_cache, void* v_cache, float* logits, w4a16_stream_t stream) {
  if (!plan || !token || !pos || !k_cache || !v_cache || !logits) {
    set_error("null pointer argument");
    return W4A16_ERR_NULL;
  }
  if (!aligned(token, 8) || !aligned(pos, 8) || !aligned(k_cache, 16) || !aligned(v_cache, 16) ||
      !aligned(logits, 4)) {
    set_error("token/pos need 8-byte, caches 16-byte, logits 4-byte alignment");
    return W4A16_ERR_ALIGN;
  }
  return w4a16::decode_step_launch(reinterpret_cast<w4a16::DecodePlan*>(plan),
                                   reinterpret_cast<const long long*>(token),
                                   reinterpret_cast<const long long*>(pos), k_cache, v_cache, logits,
                                   reinterpret_cast<cudaStream_t>(stream));
}

const char* w4a16_status_string(int status) {
  switch (status) {
    case W4A16_OK: return "ok";
    case W4A16_ERR_NULL: return "NULL pointer";
    case W4A16_ERR_SHAPE: return "bad shape";
    case W4A16_ERR_ALIGN: return "misaligned pointer";
    case W4A16_ERR_DTYPE: return "unknown dtype, packing or group";
    case W4A16_ERR_WORKSPACE: return "workspace too small";
    case W4A16_ERR_CUDA: return "CUDA error";
    case W4A16_ERR_KERNEL: return "kernel wait timed out";
    default: return "unknown status";
  }
}

const char* w4a16_last_error_string(void) { return w4a16::last_error(); }

int w4a16_version(void) { return kVersion; }

}  // extern "C"
