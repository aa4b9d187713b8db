// Internal (C++) interface between the C-ABI layer (w4a16_capi.cu) and the kernel
// launchers (w4a16_gemv.cu, w4a16_aux.cu, w4a16_decode.cu).  Nothing here crosses the
// library boundary.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

#include "w4a16_b200.h"

namespace w4a16 {

// One W4A16 product  Y[M][N] = X[M][K] . dequant(W)[N][K]^T  (+ bias), where
// dequant(W)[r][k] = (q[r][k]) * scale(r, k) and q is the signed int4 code.
struct GemvProblem {
  const uint8_t* packed = nullptr;  // [N][K/2] bytes
  int packing = W4A16_PACK_INTERLEAVED;
  const void* scale = nullptr;      // [N] (group 0) or [N][K/group]
  int scale_dtype = W4A16_DTYPE_F32;
  int group = 0;                    // 0 = one scale per row, 128 = one per 128 columns
  const void* x = nullptr;          // fp16 [M][K]
  int M = 1, N = 0, K = 0;
  void* y = nullptr;                // [M][N], dtype out_dtype
  int out_dtype = W4A16_DTYPE_F32;
  const float* bias = nullptr;      // fp32 [N] or null
  void* workspace = nullptr;        // split-K partials + tile counters (zero-filled once)
  size_t workspace_bytes = 0;
  int split_k = 0;                  // 0 = choose, 1 = no workspace schedules
  int prologue = W4A16_PROLOGUE_NONE;  // x computed from pro_src inside the kernel
  const void* pro_src = nullptr;
  const float* pro_gamma = nullptr;
  float pro_eps = 0.f;
  int tp_n = 0;                     // fused all-gather over tp_n ranks (0: plain output y)
  int tp_rank = 0;
  long long tp_row0 = 0;            // this rank's first row in the gathered output
  void* tp_out[8] = {};             // every rank's gathered output
  unsigned* tp_flags[8] = {};       // every rank's region header
  unsigned long long tp_wait_ns = 0;  // limit of each wait on another rank's flags
  bool staged = false;              // fused entry: x staged in shared memory, TMA kernel only
  bool pdl = false;                 // programmatic dependent launch (staged GEMV only)
  bool out_swiglu = false;          // gate / up row pairs per 16-row block -> silu(g) * u (RMSNorm only)
  cudaStream_t stream = nullptr;
};

// Validated launch of the W4A16 product.  Chooses the TMA/tensor-core kernel when
// the shape and alignment allow it, else the generic warp-per-row kernel.
int launch_gemv(const GemvProblem& p);

// Workspace the split-K path may use for a problem of this size.
size_t gemv_workspace_bytes(int M, int N, int K);

// Bytes at the start of a split-K workspace holding the per-tile counters, which
// must be zero when a kernel starts (the kernels leave them zeroed).
size_t gemv_counter_bytes();

// fp16 products summed in fp16 per packed word (the lossy variant), simple packing.
int launch_h2f32(const uint8_t* packed, const float* scale, const void* vec, float* out, int rows,
                 int cols, cudaStream_t stream);

// Dense fp16 matrix-vector product with fp32 accumulation (bandwidth baseline).
int launch_fp16_gemv(const void* mat, const void* vec, float* out, int rows, int cols,
                     cudaStream_t stream);

// Bit-exact dequantisation: out[r][k] = fp16(fp32(q[r][k]) * fp32(scale(r, k))).
int launch_dequant(const uint8_t* packed, int packing, const void* scale, int scale_dtype,
                   int group, int rows, int cols, void* out, cudaStream_t stream);

// Symmetric int4 quantisation + packing on the GPU (one launch):
//   scale = absmax / 7 per row or group, q = clamp(rint(w / scale), -8, 7).
int launch_quantize_pack(const void* w, int w_dtype, int rows, int cols, int group, int packing,
                         uint8_t* packed, void* scale, int scale_dtype, cudaStream_t stream);

// Decode-step attention (one token, head_dim 64) fused with rotary and the KV-cache
// write; scratch holds per-split partials and per-kv-head counters (zero-filled once).
size_t decode_attention_scratch_bytes(int heads, int kv_heads, int splits);
int launch_decode_attention(const void* qkv, const float* cos_t, const float* sin_t,
                            const long long* pos, void* k_cache, void* v_cache, void* out,
                            void* scratch, int heads, int kv_heads, int head_dim, int max_len,
                            int splits, bool pdl, cudaStream_t stream);

// Launch `kernel` with programmatic stream serialisation when `pdl` is set (the kernel
// may start while the previous one in the stream is still running; it must call
// grid_dependency_wait() before touching that kernel's outputs), normally otherwise.
template <typename... KArgs, typename... Args>
cudaError_t launch_maybe_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t stream, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Fused all-gather: bytes of the flag header at the start of every rank's region, and
// the header offset of the region's output capacity in bytes (u64, written once by
// w4a16_tp_region_alloc; the kernels use header bytes [0, 128) for their flags).
constexpr size_t kTpHeaderBytes = 256;
constexpr size_t kTpCapacityOffset = 128;
constexpr size_t kTpTimelineOffset = 192;  // 4 x u64 step stamps, written by the owner's kernel

// Reads (and clears) the device-side error word written by kernels whose bounded
// waits ran out.  Synchronises `stream`.
int read_device_error(int* code, cudaStream_t stream);

// The one-kernel decode step (w4a16_decode_step.cu): a plan holds the projection tables,
// tensor maps and the step's scratch for one model on one device.
struct DecodePlan;
int decode_plan_create(const w4a16_llama_desc* desc, DecodePlan** out);
int decode_plan_destroy(DecodePlan* plan);
int decode_step_launch(DecodePlan* plan, const long long* token, const long long* pos, void* k_cache,
                       void* v_cache, float* logits, cudaStream_t stream);
int read_decode_step_error(int* code, cudaStream_t stream);
// Tensor-core W4A16 GEMM for many activation rows (csrc/w4a16_gemm.cu); arguments checked by the caller.
int launch_gemm(const uint8_t* packed, const float* scale, int group, const void* x, const float* bias,
                int M, int N, int K, void* y, int out_dtype, void* workspace, size_t workspace_bytes,
                cudaStream_t stream);
size_t gemm_workspace_bytes(int M, int N, int K);
int read_gemm_error(int* code, cudaStream_t stream);
int decode_plan_timeline(DecodePlan* plan, int enable, unsigned long long* host, size_t capacity,
                         size_t* count, cudaStream_t stream);

// Thread-local description of the last failure, for w4a16_last_error_string().
void set_error(const char* fmt, ...);
// SM count of the current device (cached per device).
int current_sm_count(int* sms);
const char* last_error();

}  // namespace w4a16
