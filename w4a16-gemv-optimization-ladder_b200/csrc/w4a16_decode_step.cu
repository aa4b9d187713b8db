// One-kernel decode step of a Llama-architecture model on B200 (sm_100a): every layer's
// RMSNorm + QKV GEMV, rotary + KV-cache write + attention, output GEMV + residual,
// RMSNorm + gate|up GEMV, SwiGLU + down GEMV + residual, and the final norm + head GEMV,
// in one persistent launch of one CTA per SM.
//
// The reference runs a decode step as a Hugging Face model whose Linears call its GEMV
// one by one from Python (benchmarks/end_to_end.py:24-42, the swapped W4A16Linear at
// src/w4a16/kernels.py:105-124); the graph of separate kernels in w4a16/decode.py
// launches ~81 kernels per token, each paying a launch, a first-copy latency and an
// epilogue.  Here the step is a sequence of phases separated by grid-wide barriers, and
// the weights never wait for the activations:
//
//   * Work units.  Every projection is cut into (16-row tile, 1024-column window) units
//     (one TMA box each, the layout of k_gemv_tma); unit u of projection m belongs to warp
//     (u + off_m) mod W (W = warps in the grid; off_m rotates so consecutive projections
//     land on different warps).  A projection with few tiles gives each unit one window
//     and reduces a tile's windows through global partials (last arriver, window order);
//     one with many tiles gives each unit a whole tile.
//   * Look-ahead.  Every warp owns a 2-stage ring and walks its own unit stream through
//     the whole step; it issues the weight copies of its next units (of this or any later
//     projection) as soon as a stage is free, before the barrier that starts their phase,
//     so HBM streams through the barriers and most phases find their weights in place.
//   * Phases.  After each barrier every CTA stages the phase's activation vector in shared
//     memory (RMSNorm of the fp32 residual stream, the attention output, or SwiGLU of the
//     gate|up vector), then its warps consume their units of the phase.  Attention runs as
//     (kv head, 32-position split) items on the CTAs, the last split of a head combining.
//   * Barriers.  A sense-reversing counter in the plan's scratch; every wait (barrier,
//     stage, tile counter) gives up after a bounded time, records an error code and, once
//     any wait of this launch has given up, the others return at once, so a launch always
//     ends.  The grid is launched cooperatively (all CTAs resident).
//
// Numerics are those of the separate kernels: fp32 residual stream, fp16 activations into
// the GEMVs, exact int4 x fp16 products accumulated in fp32 per 128-column group, fp32
// softmax, fp16 q/k/v and attention output.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "w4a16_device.cuh"
#include "w4a16_gemv_core.cuh"
#include "w4a16_internal.h"

namespace w4a16 {

namespace {

#ifndef W4A16_DS_WARPS
#define W4A16_DS_WARPS 8
#endif
#ifndef W4A16_DS_STAGES
#define W4A16_DS_STAGES 3
#endif
// 8 warps of up to 255 registers with 3-stage rings (the same 26 KB of weights in
// flight per warp as 12 warps x 2 stages, without register spills in the window loop)
constexpr int kDsWarps = W4A16_DS_WARPS;
constexpr int kDsStages = W4A16_DS_STAGES;
constexpr int kDsSlabs = 4;
constexpr int kDsThreads = kDsWarps * 32;
constexpr int kHeadDim = 64;
constexpr int kWinCols = kDsSlabs * kSlabCols;  // 1024 columns per window
#ifndef W4A16_DS_SPAN  // slabs whose groups a warp accumulates side by side (consume_window_wide)
#define W4A16_DS_SPAN 2
#endif
constexpr int kDsSpan = W4A16_DS_SPAN;
#ifndef W4A16_DS_FILL_AT_BARRIER  // 1: local-mode copies issued only during grid barriers
#define W4A16_DS_FILL_AT_BARRIER 0
#endif
constexpr bool kDsFillAtBarrier = W4A16_DS_FILL_AT_BARRIER;
using DsL = StageLayout<kDsSlabs, 1, 128, float>;
using DsPlanLayout = SmemPlan<kDsWarps, kDsStages, DsL>;

constexpr uint64_t kDsStageWaitNs = 2000000000ull;  // a weight copy normally lands in us
constexpr uint64_t kDsSyncWaitNs = 1000000000ull;   // barriers and tile counters
constexpr uint64_t kDsDrainWaitNs = 100000000ull;

// Error codes of this kernel (w4a16_read_device_error reports them).
enum : int { kDsErrStage = 1, kDsErrBarrier = 3, kDsErrLayout = 4 };

__device__ int g_ds_error = 0;

__device__ __forceinline__ void ds_record_error(int code) { atomicCAS(&g_ds_error, 0, code); }
// A wait of this launch gave up (the error word was clear when the launch started and is
// set now); an error left by an earlier launch, not read yet, does not count.
__device__ __forceinline__ bool ds_failed(int err0) {
  return err0 == 0 && *reinterpret_cast<volatile int*>(&g_ds_error) != 0;
}

// How a projection's outputs are stored.
//   kOutSwiGlu  gate and up rows interleaved in blocks of 8 (rows 16k..16k+7 are gate
//               rows 8k..8k+7, rows 16k+8..16k+15 the matching up rows): the tile's
//               epilogue stores fp16(silu(g) * u) for its 8 rows of the MLP activation,
//               with g and u rounded to fp16 first (the separate kernels' arithmetic).
enum DsOut : int { kOutHalf = 0, kOutResidual = 1, kOutFloat = 2, kOutSwiGlu = 3 };
// How a phase's activation vector is staged.
enum DsStage : int { kStageNorm = 0, kStageCopy = 1, kStageSwiGlu = 2 };
// How a projection's work is split.
//   kModeLocal  CTA c owns the tiles of virtual CTA (c + off) mod grid (an equal contiguous
//               share); window u of the share goes to warp (u + woff) mod 12 (woff rotates
//               with the projection, so the warps that take a second window differ from
//               phase to phase), and the windows of a tile are added in shared memory, in
//               window order, once the CTA's warps are done.  For projections with at most
//               kLocalMaxWindows windows per CTA: every warp then holds at most two.
//   kModeTile   unit u (a whole tile, all its windows) belongs to warp (u + off) mod W, the
//               warps numbered warp-major over the SMs; the warp stores the tile's rows.
enum DsMode : int { kModeLocal = 0, kModeTile = 1 };
constexpr int kLocalMaxWindows = 2 * kDsWarps;

// One projection as the kernel sees it (a table in device memory, built by the plan).
struct DsMat {
  const CUtensorMap* wmap;  // 3-D view {128 B, cols/256 slabs, rows} of the packed weights
  const CUtensorMap* smap;  // 2-D view {cols/128, rows} of the fp32 group scales
  void* out;                // fp16 [rows] or fp32 [rows] (residual: out += y); the head: P.logits
  int rows, cols;
  int ntiles, nwin;         // 16-row tiles, 1024-column windows
  int mode;                 // DsMode
  int off;                  // rotation of the work over CTAs (local) or warps (tile)
  int out_kind;             // DsOut
  int woff;                 // local: rotation of the CTA's windows over its warps
  int tq, tr;               // local: tiles per CTA (ntiles = tq * grid + tr, the first tr take one more)
};
static_assert(sizeof(DsMat) % 16 == 0, "the table is copied to shared memory in 16-byte pieces");

struct DsParams {
  const DsMat* mats;           // [4 * layers + 1]: per layer qkv, o, gate|up, down; then the head
  const float* const* norms;   // [2 * layers + 1]: attention norm, MLP norm per layer; final norm
  const __half* embed;         // [vocab][hidden]
  const float* cos_t;          // [max_len][64] rotate-half tables
  const float* sin_t;
  const long long* token;      // device int64 [1]
  const long long* pos;        // device int64 [1]
  __half* k_cache;             // [layers][kv_heads][max_len][64]
  __half* v_cache;
  float* h;                    // [hidden] residual stream
  __half* qkv;                 // [(heads + 2 kv_heads) * 64]
  __half* attn;                // [heads * 64]
  __half* gu;                  // [2 * intermediate]
  float* logits;               // [vocab], the head's output
  float* attn_part;            // [heads][splits][66]
  unsigned* attn_cnt;          // [kv_heads], zero between uses
  unsigned long long* bar;     // grid-barrier arrivals, monotonic over the plan's steps
  int layers, hidden, inter, heads, kv_heads, max_len, splits, nmats, vocab;
  int gu_interleaved;          // gate|up rows interleaved by 8: P.gu holds the activation [inter]
  int kv_off;                  // shared-memory offset (in the x area) of the attention rows
  int lpart_off, table_off;    // shared-memory offsets (from the x area) of the local partials and table
  int xbytes;                  // shared-memory bytes of the staged vector / attention state
  float eps;
  // optional timeline, [3 * (barriers + 1)][grid] %globaltimer ns per CTA: start, end and
  // the first phase's staged vector, then for every grid barrier the arrival, the
  // departure and the staged vector of the phase after it
  unsigned long long* stamps;
};

__device__ __forceinline__ float ds_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float ds_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Grid-wide barrier on a monotonic arrival counter: barrier k of a step (k = 1, 2, ...)
// is passed once the counter reaches base + k * grid, where base is the counter at the
// start of the step (every step adds exactly barriers * grid).  One release-add per CTA,
// then polling with acquire loads: a single L2 round trip after the last arrival.
// `meanwhile` runs on every thread between the CTA's arrival and its wait (the warps
// issue their next weight copies there, off the critical path).  Bounded: a wait that runs
// out records kDsErrBarrier; once any wait of the launch has failed, the barrier returns
// at once.
template <typename Meanwhile>
__device__ __forceinline__ void ds_grid_barrier(unsigned long long* bar, unsigned long long base, int err0,
                                                unsigned long long* stamps, int& nbar, Meanwhile&& meanwhile) {
  __syncthreads();
  ++nbar;
  const unsigned long long target = base + (unsigned long long)nbar * gridDim.x;
  if (threadIdx.x == 0) {
    if (stamps) stamps[(size_t)(3 * nbar) * gridDim.x + blockIdx.x] = globaltimer_ns();
    red_release_gpu_add_u64(bar, 1ull);
  }
  meanwhile();
  if (threadIdx.x == 0) {
    if (ld_acquire_gpu_u64(bar) < target) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_gpu_u64(bar) < target) {
        if (ds_failed(err0)) break;
        if (globaltimer_ns() - t0 > kDsSyncWaitNs) {
          ds_record_error(kDsErrBarrier);
          break;
        }
      }
    }
    if (stamps) stamps[(size_t)(3 * nbar + 1) * gridDim.x + blockIdx.x] = globaltimer_ns();
  }
  __syncthreads();
}

// Read-only load of a pointer field of the (kernel-constant) tables.
template <typename T>
__device__ __forceinline__ T ldg_ptr(const T* p) {
  return reinterpret_cast<T>(__ldg(reinterpret_cast<const unsigned long long*>(p)));
}

__device__ __forceinline__ int ds_mod(int a, int w) {
  const int r = a % w;
  return r < 0 ? r + w : r;
}

// This warp's share of projection m.
//   local: units u0, u0 + 12, ... < u1 of the CTA's share (tiles [tb0, tb0 + ntl)), one
//          window each
//   tile:  units u0, u0 + W, ... < u1 (= ntiles), one tile each
struct DsShare {
  int u0, u1, tb0, ntl;
};

__device__ __forceinline__ DsShare ds_share(const DsMat* m, int W, int gw, int warp) {
  DsShare sh;
  const int ntiles = m->ntiles;
  if (m->mode == kModeLocal) {
    const int vc = ds_mod((int)blockIdx.x + m->off, (int)gridDim.x);
    const int q = m->tq, r = m->tr;
    sh.tb0 = vc * q + min(vc, r);
    sh.ntl = q + (vc < r ? 1 : 0);
    sh.u0 = ds_mod(warp - m->woff, kDsWarps);
    sh.u1 = sh.ntl * m->nwin;
  } else {
    sh.tb0 = 0;
    sh.ntl = 0;
    sh.u0 = ds_mod(gw - m->off, W);
    sh.u1 = ntiles;
  }
  return sh;
}

// Position in a warp's unit stream: projection mi, unit u (with its share).
struct DsCursor {
  int mi, u;
  DsShare sh;
};

__device__ __forceinline__ void ds_seek(const DsMat* mats, int nmats, int W, int gw, int warp, DsCursor& c) {
  while (c.mi < nmats) {
    c.sh = ds_share(mats + c.mi, W, gw, warp);
    c.u = c.sh.u0;
    if (c.u < c.sh.u1) return;
    ++c.mi;
  }
}

__device__ __forceinline__ void ds_advance(const DsMat* mats, int nmats, int W, int gw, int warp, DsCursor& c) {
  c.u += mats[c.mi].mode == kModeLocal ? kDsWarps : W;
  if (c.u < c.sh.u1) return;
  ++c.mi;
  ds_seek(mats, nmats, W, gw, warp, c);
}

// fence the tensor maps written by the host before their first use by the TMA unit
__device__ __forceinline__ void tensormap_acquire(const void* map) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(map) : "memory");
}

// Stage the activation vector of a phase into shared memory (fragment order), and the
// group corrections of the folded decode: corr[grp] = -72 * (sum of x over columns
// 8i+2, 8i+3, 8i+6, 8i+7 of the group).  Every load of a thread is issued before the
// first is used (one L2 round trip).
constexpr int kChunks = 4;  // 8-element chunks per thread in the copy / SwiGLU stages
constexpr int kMaxStageK = kChunks * 8 * kDsThreads;  // their largest vector
constexpr int kMaxNormK = 2 * 8 * kDsThreads;         // the RMSNorm stage's largest vector

__device__ __forceinline__ void ds_fold_correction(float* corr_f, int lane, int c, int nch, const uint4& v) {
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.w));
  float part = (a.x + a.y) + (b.x + b.y);
#pragma unroll
  for (int o = 1; o < 16; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if ((lane & 15) == 0 && c < nch) corr_f[c >> 4] = -72.f * part;
}

__device__ __forceinline__ void ds_put(uint8_t* xsp, int c, const uint4& o) {
  *reinterpret_cast<uint4*>(xsp + xs_offset(c * 8)) = o;
}

// RMSNorm of the residual stream (or, for the first layer, of the embedding row):
// K <= kMaxNormK (the hidden size), two chunks per thread at most.
__device__ __noinline__ void ds_stage_norm(const DsParams& P, int K, const float* gamma, const __half* erow,
                                         uint8_t* xsp, float* redp, float* corr_f) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool from_embed = erow != nullptr;
  const int nch = K >> 3;
  float v[2][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int c = threadIdx.x + j * kDsThreads;
    if (c < nch) {
      if (from_embed) {
        const uint4 e = ldg128(erow + c * 8);
        const uint32_t ew[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ew[i]));
          v[j][2 * i] = f.x;
          v[j][2 * i + 1] = f.y;
        }
      } else {
        const float4 a = __ldcg(reinterpret_cast<const float4*>(P.h) + 2 * c);
        const float4 b = __ldcg(reinterpret_cast<const float4*>(P.h) + 2 * c + 1);
        v[j][0] = a.x; v[j][1] = a.y; v[j][2] = a.z; v[j][3] = a.w;
        v[j][4] = b.x; v[j][5] = b.y; v[j][6] = b.z; v[j][7] = b.w;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(v[j][i], v[j][i], ss);
    }
  }
  ss = ds_warp_sum(ss);
  if (lane == 0) redp[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kDsWarps; ++w) tot += redp[w];
  const float r = rsqrtf(tot / (float)K + P.eps);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int c = threadIdx.x + j * kDsThreads;
    if (j * kDsThreads >= nch) break;  // warp-uniform (nch is a multiple of 32)
    uint4 o = make_uint4(0u, 0u, 0u, 0u);
    if (c < nch) {
      const float4 ga = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * c);
      const float4 gb = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * c + 1);
      o.x = pack_half2(v[j][0] * r * ga.x, v[j][1] * r * ga.y);
      o.y = pack_half2(v[j][2] * r * ga.z, v[j][3] * r * ga.w);
      o.z = pack_half2(v[j][4] * r * gb.x, v[j][5] * r * gb.y);
      o.w = pack_half2(v[j][6] * r * gb.z, v[j][7] * r * gb.w);
      ds_put(xsp, c, o);
    }
    ds_fold_correction(corr_f, lane, c, nch, o);
  }
  __syncthreads();
}

__device__ __noinline__ void ds_stage_copy(int K, const __half* src, uint8_t* xsp, float* corr_f) {
  const int lane = threadIdx.x & 31;
  const int nch = K >> 3;
  uint4 o[kChunks];
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    const int c = threadIdx.x + j * kDsThreads;
    o[j] = c < nch ? ldcg128(src + c * 8) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    const int c = threadIdx.x + j * kDsThreads;
    if (j * kDsThreads >= nch) break;
    if (c < nch) ds_put(xsp, c, o[j]);
    ds_fold_correction(corr_f, lane, c, nch, o[j]);
  }
  __syncthreads();
}

__device__ __noinline__ void ds_stage_swiglu(int K, const __half* src, uint8_t* xsp, float* corr_f) {
  const int lane = threadIdx.x & 31;
  const int nch = K >> 3;
  uint4 gv[kChunks], uv[kChunks];
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    const int c = threadIdx.x + j * kDsThreads;
    gv[j] = c < nch ? ldcg128(src + c * 8) : make_uint4(0u, 0u, 0u, 0u);
    uv[j] = c < nch ? ldcg128(src + K + c * 8) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    const int c = threadIdx.x + j * kDsThreads;
    if (j * kDsThreads >= nch) break;
    uint4 o = make_uint4(0u, 0u, 0u, 0u);
    if (c < nch) {
      const uint32_t gw4[4] = {gv[j].x, gv[j].y, gv[j].z, gv[j].w};
      const uint32_t uw4[4] = {uv[j].x, uv[j].y, uv[j].z, uv[j].w};
      uint32_t pk[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 g2 = __half22float2(*reinterpret_cast<const __half2*>(&gw4[i]));
        const float2 u2 = __half22float2(*reinterpret_cast<const __half2*>(&uw4[i]));
        pk[i] = pack_half2(g2.x / (1.0f + expf(-g2.x)) * u2.x, g2.y / (1.0f + expf(-g2.y)) * u2.y);
      }
      o = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      ds_put(xsp, c, o);
    }
    ds_fold_correction(corr_f, lane, c, nch, o);
  }
  __syncthreads();
}


// Attention chunks: a chunk is 32 positions of one kv head (one item); its key and value
// rows below pos were written by earlier steps, so the CTA owning the item copies them into
// shared memory (two bulk copies) at the start of the layer's QKV phase, off the critical
// path; the attention phase then reads them there.
constexpr int kAttnSpan = 32;

struct DsAttnSmem {
  uint32_t kv;    // shared address of [K rows | V rows] of the chunk, 2 * 32 * 128 bytes
  uint32_t bar;   // its mbarrier
};

// Issue the copy of this CTA's first attention item of layer `layer`; returns whether one
// was issued (the attention phase then waits for it).
__device__ __forceinline__ bool ds_load_attention_kv(const DsParams& P, int layer, int pos, const DsAttnSmem& a) {
  const int item = blockIdx.x;
  if (item >= P.kv_heads * P.splits) return false;
  const int kvh = item / P.splits;
  const int c0 = (item - kvh * P.splits) * kAttnSpan;
  const int c1 = min(c0 + kAttnSpan, pos);  // rows [c0, c1); the row at pos is written this step
  if (c1 <= c0) return false;
  if (threadIdx.x == 0) {
    const size_t off = (((size_t)layer * P.kv_heads + kvh) * P.max_len + c0) * kHeadDim;
    const uint32_t bytes = (uint32_t)(c1 - c0) * kHeadDim * 2;
    fence_proxy_async_smem();  // the region held the previous phase's staged vector
    mbar_arrive_expect_tx(a.bar, 2 * bytes);
    bulk_load(a.kv, P.k_cache + off, bytes, a.bar);
    bulk_load(a.kv + kAttnSpan * kHeadDim * 2, P.v_cache + off, bytes, a.bar);
  }
  return true;
}

// Attention of layer `layer` for one token.  Item i (kv head, 32-position chunk) runs on
// CTA i (and i + grid, ...): warp w takes query head w % group of the kv head's group and
// the 32 / (warps / group) positions of slice w / group of the chunk; the slices of a head
// are combined in shared memory, the chunk's partial softmax (max, sum, unnormalised
// output) goes to global memory, and the last chunk of a kv head to finish combines the
// chunks in order.  kv_ready: this CTA's first item has its rows in shared memory (after
// waiting for kv_parity of a.bar).
__device__ __noinline__ void ds_attention(const DsParams& P, int layer, int pos, bool bad_pos, uint8_t* xsp,
                                          unsigned* s_prev, DsAttnSmem a, bool kv_ready, uint32_t kv_parity,
                                          int err0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int max_len = P.max_len;
  const int group = P.heads / P.kv_heads;
  const int slices = kDsWarps / group;       // position slices per chunk
  const int slen = kAttnSpan / slices;       // positions per slice (<= 32)
  const int splits = P.splits;               // chunks per kv head: ceil(max_len / 32)
  const float scale = 0.125f;                // 1 / sqrt(64)
  constexpr int kPart = kHeadDim + 2;
  float* qs = reinterpret_cast<float*>(xsp);   // [group][64] rotated, scaled queries
  float* kn = qs + group * kHeadDim;           // [64] new key, [64] new value
  float* vn = kn + kHeadDim;
  float* bp = vn + kHeadDim;                   // [warps][66] per-slice partials
  const int hq = warp % group;
  const int sl = warp / group;
  const bool active = warp < group * slices && !bad_pos;
  if (kv_ready && !mbar_wait_bounded(a.bar, kv_parity, kDsStageWaitNs)) {
    ds_record_error(kDsErrStage);
    kv_ready = false;  // read the rows from global memory instead
  }
  for (int item = blockIdx.x; item < P.kv_heads * splits; item += gridDim.x) {
    const bool in_smem = kv_ready && item == (int)blockIdx.x;
    const int kvh = item / splits;
    const int split = item - kvh * splits;
    const int c0 = split * kAttnSpan;
    const size_t cache_off = ((size_t)layer * P.kv_heads + kvh) * max_len * kHeadDim;
    __half* kc = P.k_cache + cache_off;
    __half* vc = P.v_cache + cache_off;
    const float* cr = P.cos_t + (size_t)pos * kHeadDim;
    const float* sr = P.sin_t + (size_t)pos * kHeadDim;
    const int head = kvh * group + hq;
    if (active && sl == 0) {  // rotate query head hq of the group
      const float qa = __half2float(__ldcg(P.qkv + head * kHeadDim + lane));
      const float qb = __half2float(__ldcg(P.qkv + head * kHeadDim + lane + 32));
      qs[hq * kHeadDim + lane] = (qa * cr[lane] - qb * sr[lane]) * scale;
      qs[hq * kHeadDim + lane + 32] = (qb * cr[lane + 32] + qa * sr[lane + 32]) * scale;
    }
    if (warp == kDsWarps - 1 && !bad_pos && pos >= c0 && pos < c0 + kAttnSpan) {
      // this chunk owns the new position: the rotated key and the value go into the cache
      const int kb = P.heads * kHeadDim + kvh * kHeadDim;
      const int vb = (P.heads + P.kv_heads) * kHeadDim + kvh * kHeadDim;
      const float ka = __half2float(__ldcg(P.qkv + kb + lane));
      const float kb2 = __half2float(__ldcg(P.qkv + kb + lane + 32));
      const __half ah = __float2half_rn(ka * cr[lane] - kb2 * sr[lane]);
      const __half bh = __float2half_rn(kb2 * cr[lane + 32] + ka * sr[lane + 32]);
      const __half va = __ldcg(P.qkv + vb + lane), vb2 = __ldcg(P.qkv + vb + lane + 32);
      kc[(size_t)pos * kHeadDim + lane] = ah;
      kc[(size_t)pos * kHeadDim + lane + 32] = bh;
      vc[(size_t)pos * kHeadDim + lane] = va;
      vc[(size_t)pos * kHeadDim + lane + 32] = vb2;
      kn[lane] = __half2float(ah);
      kn[lane + 32] = __half2float(bh);
      vn[lane] = __half2float(va);
      vn[lane + 32] = __half2float(vb2);
    }
    __syncthreads();
    if (active) {  // slice sl of the chunk for head hq: positions [jb, jb + nv) of [0, pos]
      const int jb = c0 + sl * slen;
      const int j1 = min(min(jb + slen, max_len), pos + 1);
      const int nv = max(0, j1 - jb);
      float m = -INFINITY, l = 0.f;
      float2 o = make_float2(0.f, 0.f);
      if (nv > 0) {
        const float* q = qs + hq * kHeadDim;
        // score of position jb + (lane % slen): the lanes of one position split the 64 dims
        const int lanes_per_pos = 32 / slen;
        const int pi = lane % slen;
        const int part = lane / slen;             // dims [part * 64 / lanes_per_pos, ...)
        const int dlen = kHeadDim / lanes_per_pos;
        const int jj = jb + pi;
        float d = 0.f;
        if (pi < nv) {
          if (jj == pos) {
            for (int e = part * dlen; e < (part + 1) * dlen; ++e) d = fmaf(q[e], kn[e], d);
          } else {
            const __half* krow = in_smem ? nullptr : kc + (size_t)jj * kHeadDim;
            const uint32_t ksm = a.kv + (uint32_t)(jj - c0) * kHeadDim * 2;
            // 16-byte pieces of the row, started at a lane-dependent piece (no bank conflicts)
            const int pieces = dlen / 8;
            for (int k = 0; k < pieces; ++k) {
              const int pc = part * pieces + (k + pi) % pieces;
              const uint4 kv = in_smem ? lds128(ksm + pc * 16) : *reinterpret_cast<const uint4*>(krow + pc * 8);
              const uint32_t w4[4] = {kv.x, kv.y, kv.z, kv.w};
              const float4 qa = *reinterpret_cast<const float4*>(q + pc * 8);
              const float4 qb = *reinterpret_cast<const float4*>(q + pc * 8 + 4);
              const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
                d = fmaf(qv[2 * i], f.x, d);
                d = fmaf(qv[2 * i + 1], f.y, d);
              }
            }
          }
        }
        for (int o2 = slen; o2 < 32; o2 <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o2);  // add the dim parts
        const float sc = pi < nv ? d : -INFINITY;
        m = ds_warp_max(sc);
        const float pj = sc == -INFINITY ? 0.f : __expf(sc - m);
        l = ds_warp_sum(pj) / (float)lanes_per_pos;  // every position was counted lanes_per_pos times
        // output dims (2 lane, 2 lane + 1): value rows of the slice
        for (int u = 0; u < nv; ++u) {
          const float pu = __shfl_sync(0xffffffffu, pj, u);
          float2 v;
          if (jb + u == pos) {
            v = make_float2(vn[2 * lane], vn[2 * lane + 1]);
          } else if (in_smem) {
            const uint32_t vsm = a.kv + kAttnSpan * kHeadDim * 2 + (uint32_t)(jb + u - c0) * kHeadDim * 2;
            uint32_t w;
            asm volatile("ld.shared.b32 %0, [%1];" : "=r"(w) : "r"(vsm + lane * 4));
            v = __half22float2(*reinterpret_cast<const __half2*>(&w));
          } else {
            v = __half22float2(reinterpret_cast<const __half2*>(vc + (size_t)(jb + u) * kHeadDim)[lane]);
          }
          o.x = fmaf(pu, v.x, o.x);
          o.y = fmaf(pu, v.y, o.y);
        }
      }
      float* mine = bp + warp * kPart;
      if (lane == 0) {
        mine[0] = m;
        mine[1] = l;
      }
      reinterpret_cast<float2*>(mine + 2)[lane] = o;
    }
    __syncthreads();
    if (active && sl == 0) {  // combine head hq's slices, write the chunk's partial
      float M = -INFINITY;
      for (int b = 0; b < slices; ++b) M = fmaxf(M, bp[(b * group + hq) * kPart]);
      float L = 0.f;
      float2 acc = make_float2(0.f, 0.f);
      for (int b = 0; b < slices; ++b) {
        const float* pb = bp + (b * group + hq) * kPart;
        if (pb[0] == -INFINITY) continue;
        const float w = __expf(pb[0] - M);
        L += pb[1] * w;
        const float2 ob = reinterpret_cast<const float2*>(pb + 2)[lane];
        acc.x = fmaf(ob.x, w, acc.x);
        acc.y = fmaf(ob.y, w, acc.y);
      }
      float* part = P.attn_part + ((size_t)head * splits + split) * kPart;
      if (lane == 0) {
        __stcg(part, M);
        __stcg(part + 1, L);
      }
      __stcg(reinterpret_cast<float2*>(part + 2) + lane, acc);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *s_prev = atomicAdd(P.attn_cnt + kvh, 1u);
    __syncthreads();
    if (*s_prev == (unsigned)(splits - 1)) {  // the last chunk of this kv head combines
      __threadfence();
      if (warp < group) {
        const int hd = kvh * group + warp;
        const float* ph = P.attn_part + (size_t)hd * splits * kPart;
        if (bad_pos) {
          reinterpret_cast<__half2*>(P.attn + hd * kHeadDim)[lane] = __float2half2_rn(__int_as_float(0x7fc00000));
        } else {
          // chunks past pos hold nothing; lane s < 32 loads chunk s's max and sum, and every
          // lane its two dims of each chunk's output
          const int nsplit = min(splits, pos / kAttnSpan + 1);
          float M = -INFINITY;
          for (int s0 = 0; s0 < nsplit; s0 += 32)
            if (s0 + lane < nsplit) M = fmaxf(M, __ldcg(ph + (size_t)(s0 + lane) * kPart));
          M = ds_warp_max(M);
          float L = 0.f;
          float2 acc = make_float2(0.f, 0.f);
          for (int s0 = 0; s0 < nsplit; s0 += 32) {
            const int sidx = s0 + lane;
            float w = 0.f, lw = 0.f;
            if (sidx < nsplit) {
              const float ms = __ldcg(ph + (size_t)sidx * kPart);
              w = ms == -INFINITY ? 0.f : __expf(ms - M);
              lw = __ldcg(ph + (size_t)sidx * kPart + 1) * w;
            }
            for (int u0 = 0; u0 < 32 && s0 + u0 < nsplit; u0 += 8) {
              float2 os[8];
#pragma unroll
              for (int u = 0; u < 8; ++u)
                if (s0 + u0 + u < nsplit)
                  os[u] = __ldcg(reinterpret_cast<const float2*>(ph + (size_t)(s0 + u0 + u) * kPart + 2) + lane);
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const float wu = __shfl_sync(0xffffffffu, w, u0 + u);
                const float lu = __shfl_sync(0xffffffffu, lw, u0 + u);
                if (s0 + u0 + u < nsplit) {
                  L += lu;
                  acc.x = fmaf(os[u].x, wu, acc.x);
                  acc.y = fmaf(os[u].y, wu, acc.y);
                }
              }
            }
          }
          reinterpret_cast<__half2*>(P.attn + hd * kHeadDim)[lane] = __floats2half2_rn(acc.x / L, acc.y / L);
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) P.attn_cnt[kvh] = 0u;
    }
    __syncthreads();
  }
  (void)err0;
}

__global__ void __launch_bounds__(kDsThreads, 1) k_decode_step(const __grid_constant__ DsParams P) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  uint8_t* const sbase_ptr = smem_raw + (base - smem_addr(smem_raw));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int t = lane & 3;
  const int W = gridDim.x * kDsWarps;
  const int gw = warp * gridDim.x + blockIdx.x;  // warp-major: tile-mode units spread over SMs
  const int nmats = P.nmats;

  // shared memory: [rings][scales][mbarriers][x staging | attention state: xbytes]
  // [128 B scratch][group corrections: kmax / 128 floats, 128-byte padded][local partial
  // sums][projection table]
  const uint32_t wring = base + (uint32_t)(warp * kDsStages * DsL::kWStride);
  const uint32_t sring = base + (uint32_t)(DsPlanLayout::kScaleOff + warp * kDsStages * DsL::kSStride);
  const uint32_t bar0 = base + (uint32_t)(DsPlanLayout::kBarOff + warp * kDsStages * 8);
  const uint32_t xs = base + (uint32_t)DsPlanLayout::kXOff;
  const int xbytes = P.xbytes;
  const uint32_t corr = xs + (uint32_t)xbytes + 128u;
  uint8_t* xsp = sbase_ptr + DsPlanLayout::kXOff;
  float* redp = reinterpret_cast<float*>(xsp + xbytes);
  float* corr_f = redp + 32;
  // [local partials: kLocalMaxWindows x 16 floats][projection table], 128-byte aligned
  // offsets from the plan (the corrections before them take kmax / 128 floats)
  float* lpart = reinterpret_cast<float*>(xsp + P.lpart_off);
  // the projection table, copied from global memory: the unit streams read it on every step
  DsMat* mats = reinterpret_cast<DsMat*>(xsp + P.table_off);
  if ((P.table_off | P.lpart_off | P.kv_off | P.xbytes) & 127) {  // the plan keeps them 128-aligned
    if (threadIdx.x == 0) ds_record_error(kDsErrLayout);
    return;  // every CTA returns here: no barrier is left waiting
  }
  for (int i = threadIdx.x; i < nmats * (int)(sizeof(DsMat) / 16); i += blockDim.x)
    reinterpret_cast<uint4*>(mats)[i] = __ldg(reinterpret_cast<const uint4*>(P.mats) + i);
  __shared__ unsigned s_prev;
  DsAttnSmem attn_sm;  // attention rows of this CTA's first item: [K | V] at kv_off, mbarrier in the scratch
  attn_sm.kv = xs + (uint32_t)P.kv_off;
  attn_sm.bar = xs + (uint32_t)xbytes + 120u;

  const int err0 = *reinterpret_cast<volatile int*>(&g_ds_error);
  // the barrier counter at the start of this step (no CTA can pass barrier 1 before every
  // CTA has read it, and a step adds barriers * grid)
  const unsigned long long per_step = (unsigned long long)P.layers * 5ull * gridDim.x;
  const unsigned long long bar_base = ld_acquire_gpu_u64(P.bar) / per_step * per_step;
  if (lane == 0) {
    for (int s = 0; s < kDsStages; ++s) mbar_init(bar0 + 8 * s, 1);
    if (warp == 0) mbar_init(attn_sm.bar, 1);
    mbar_fence_init();
  }
  for (int i = threadIdx.x; i < 2 * nmats; i += blockDim.x) {
    const DsMat* m = P.mats + (i >> 1);
    const void* map = (i & 1) ? (const void*)ldg_ptr(&m->smap) : (const void*)ldg_ptr(&m->wmap);
    tensormap_acquire(map);
    tma_prefetch_desc(static_cast<const CUtensorMap*>(map));
  }
  __syncthreads();
  const uint64_t policy = l2_policy_evict_first();
  const LaneOffsets lo = lane_offsets(g, t);

  // ---- producer: this warp's unit stream over the whole step, one window per stage
  DsCursor pc;
  pc.mi = 0;
  ds_seek(mats, nmats, W, gw, warp, pc);
  int p_wi = 0;
  int issued = 0, consumed = 0;
  bool stage_failed = false;
  auto issue_one = [&]() {
    if (pc.mi >= nmats || issued - consumed >= kDsStages) return;
    const DsMat* m = mats + pc.mi;
    const bool local = m->mode == kModeLocal;
    const int nwin = m->nwin;
    const int tile = local ? pc.sh.tb0 + pc.u / nwin : pc.u;
    const int win = local ? pc.u - (pc.u / nwin) * nwin : p_wi;
    if (lane == 0) {
      const uint32_t slot = (uint32_t)issued % kDsStages;
      const uint32_t bar = bar0 + 8 * slot;
      mbar_arrive_expect_tx(bar, (uint32_t)(DsL::kWBytes + DsL::kSBytes));
      tma_load_3d(wring + slot * DsL::kWStride, m->wmap, 0, win * kDsSlabs, tile * kMmaRows, bar, policy);
      tma_load_2d(sring + slot * DsL::kSStride, m->smap, win * DsL::kGroups, tile * kMmaRows, bar, policy);
    }
    ++issued;
    if (local || ++p_wi == nwin) {
      p_wi = 0;
      ds_advance(mats, nmats, W, gw, warp, pc);
    }
  };
  // every free stage of this warp's ring gets its next window (at kernel start and during
  // the grid barriers; between them a warp refills a stage as soon as it has consumed it)
  auto fill_rings = [&]() {
    if (!stage_failed)
      for (int s = 0; s < kDsStages; ++s) issue_one();
    // the descriptors of the projection this warp's copies come from next, into the TMA
    // unit's cache before the copies are issued
    if (lane == 0 && pc.mi < nmats) {
      tma_prefetch_desc(mats[pc.mi].wmap);
      tma_prefetch_desc(mats[pc.mi].smap);
    }
  };

  // ---- consumer position (the same stream)
  DsCursor cc;
  cc.mi = 0;
  ds_seek(mats, nmats, W, gw, warp, cc);

  // A position outside the cache or a token outside the vocabulary: nothing is read out of
  // bounds or written to the cache, and the attention outputs (hence the logits) are NaN.
  const long long pos_ll = *P.pos;
  const long long tok_ll = *P.token;
  const int max_len = P.max_len;
  const bool bad_tok = tok_ll < 0 || tok_ll >= P.vocab;
  const bool bad_pos = pos_ll < 0 || pos_ll >= max_len || bad_tok;
  const int pos = bad_pos ? 0 : (int)pos_ll;
  const __half* erow = P.embed + (size_t)(bad_tok ? 0 : tok_ll) * P.hidden;

  // One output row of projection m.
  auto store_row = [&](const DsMat* m, int r, float v) {
    const int kind = m->out_kind;
    void* out = m->out;
    if (kind == kOutHalf) {
      static_cast<__half*>(out)[r] = __float2half_rn(v);
    } else if (kind == kOutResidual) {
      float* hp = static_cast<float*>(out);
      hp[r] = __ldcg(hp + r) + v;
    } else {
      P.logits[r] = v;
    }
  };

  // The activation of one (gate, up) row pair of an interleaved gate|up projection.
  auto store_act = [&](const DsMat* m, int row_pair, float vg, float vu) {
    const float gg = __half2float(__float2half_rn(vg));
    const float uu = __half2float(__float2half_rn(vu));
    static_cast<__half*>(m->out)[row_pair] = __float2half_rn(gg / (1.0f + expf(-gg)) * uu);
  };

  // Consume this warp's units of projection mi (staged vector in xs, corrections in corr).
  // Local mode: window partials go to lpart and the CTA adds them at the end.
  auto run_projection = [&](int mi) {
    const DsMat* m = mats + mi;
    const bool local = m->mode == kModeLocal;
    const int nwin = m->nwin;
    const int rows = m->rows;
    const bool swiglu = m->out_kind == kOutSwiGlu;
    while (cc.mi == mi) {
      const int tile = local ? cc.sh.tb0 + cc.u / nwin : cc.u;
      const int w0 = local ? cc.u - (cc.u / nwin) * nwin : 0;
      const int nw = local ? 1 : nwin;
      float tot[1][1][4] = {{{0.f, 0.f, 0.f, 0.f}}};
      for (int wi = 0; wi < nw; ++wi) {
        const int win = w0 + wi;
        const uint32_t slot = (uint32_t)consumed % kDsStages;
        const uint32_t parity = ((uint32_t)consumed / kDsStages) & 1u;
        if (!stage_failed && !mbar_wait_bounded(bar0 + 8 * slot, parity, kDsStageWaitNs)) {
          // a copy that did not land: record it, let every copy still in flight land (or
          // give up on it) and issue nothing more in this launch
          ds_record_error(kDsErrStage);
          for (int s2 = consumed + 1; s2 < issued; ++s2)
            mbar_wait_bounded(bar0 + 8 * (s2 % kDsStages), (s2 / kDsStages) & 1u, kDsDrainWaitNs);
          stage_failed = true;
        }
        if (!stage_failed) {
          const uint32_t wb = wring + slot * DsL::kWStride;
          const uint32_t sb = sring + slot * DsL::kSStride;
          // every window is full: the plan takes column counts that are multiples of 1024
          consume_window_wide<kDsSpan, float>(wb, sb, xs, corr, win * kWinCols, g, lo, tot[0][0]);
        }
        __syncwarp();
        ++consumed;
        if ((!local || !kDsFillAtBarrier) && !stage_failed) issue_one();
      }
      // rows g and g + 8 of the tile are in tot[0][0][0] / [2] of the lanes with t == 0
      if (t == 0) {
        if (local) {
          lpart[cc.u * kMmaRows + g] = tot[0][0][0];
          lpart[cc.u * kMmaRows + g + 8] = tot[0][0][2];
        } else if (swiglu) {  // gate row g, up row g + 8 (rows are a multiple of 16)
          store_act(m, tile * 8 + g, tot[0][0][0], tot[0][0][2]);
        } else {
          const int r0 = tile * kMmaRows + g;
          if (r0 < rows) store_row(m, r0, tot[0][0][0]);
          if (r0 + 8 < rows) store_row(m, r0 + 8, tot[0][0][2]);
        }
      }
      ds_advance(mats, nmats, W, gw, warp, cc);
    }
    if (local && swiglu) {  // add each tile's windows in window order; store its 8 activations
      __syncthreads();
      const DsShare sh = ds_share(m, W, gw, warp);
      for (int i = threadIdx.x; i < sh.ntl * 8; i += blockDim.x) {
        const int tl = i >> 3, row = i & 7;
        float vg = 0.f, vu = 0.f;
        for (int w = 0; w < nwin; ++w) {
          vg += lpart[(tl * nwin + w) * kMmaRows + row];
          vu += lpart[(tl * nwin + w) * kMmaRows + row + 8];
        }
        store_act(m, (sh.tb0 + tl) * 8 + row, vg, vu);
      }
    } else if (local) {  // add each tile's windows in window order and store its rows
      __syncthreads();
      const DsShare sh = ds_share(m, W, gw, warp);
      for (int i = threadIdx.x; i < sh.ntl * kMmaRows; i += blockDim.x) {
        const int tl = i / kMmaRows, row = i - tl * kMmaRows;
        float v = 0.f;
        for (int w = 0; w < nwin; ++w) v += lpart[(tl * nwin + w) * kMmaRows + row];
        const int r = (sh.tb0 + tl) * kMmaRows + row;
        if (r < rows) store_row(m, r, v);
      }
    }
  };

  fill_rings();

  // ---- the step
  int nbar = 0;  // barriers passed (timeline index)
  int kv_uses = 0;  // attention copies issued (their mbarrier's completed phases)
  auto staged = [&]() {  // timeline: the phase's vector is in shared memory
    if (P.stamps && threadIdx.x == 0) P.stamps[(size_t)(3 * nbar + 2) * gridDim.x + blockIdx.x] = globaltimer_ns();
  };
  if (P.stamps && threadIdx.x == 0) P.stamps[blockIdx.x] = globaltimer_ns();  // slot 0: start
  if (blockIdx.x == 0) {  // the residual stream starts as the token's embedding row
    for (int i = threadIdx.x; i < P.hidden; i += blockDim.x) P.h[i] = __half2float(erow[i]);
  }
  const int qk = P.heads * kHeadDim;
  for (int layer = 0; layer < P.layers; ++layer) {
    const int mb = layer * 4;
    if (layer > 0) ds_grid_barrier(P.bar, bar_base, err0, P.stamps, nbar, fill_rings);
    // this layer's attention rows start coming into shared memory now
    const bool kv_ready = !bad_pos && ds_load_attention_kv(P, layer, pos, attn_sm);
    if (kv_ready) ++kv_uses;
    ds_stage_norm(P, P.hidden, P.norms[2 * layer], layer == 0 ? erow : nullptr, xsp, redp, corr_f);
    staged();
    run_projection(mb + 0);  // qkv = W_qkv rmsnorm(h)
    ds_grid_barrier(P.bar, bar_base, err0, P.stamps, nbar, fill_rings);
    staged();
    // attn = attention(rotary(q, k), cache)
    ds_attention(P, layer, pos, bad_pos, xsp, &s_prev, attn_sm, kv_ready, (uint32_t)(kv_uses - 1) & 1u, err0);
    ds_grid_barrier(P.bar, bar_base, err0, P.stamps, nbar, fill_rings);
    ds_stage_copy(qk, P.attn, xsp, corr_f);
    staged();
    run_projection(mb + 1);  // h += W_o attn
    ds_grid_barrier(P.bar, bar_base, err0, P.stamps, nbar, fill_rings);
    ds_stage_norm(P, P.hidden, P.norms[2 * layer + 1], nullptr, xsp, redp, corr_f);
    staged();
    run_projection(mb + 2);  // gu = W_gu rmsnorm(h)
    ds_grid_barrier(P.bar, bar_base, err0, P.stamps, nbar, fill_rings);
    if (P.gu_interleaved)
      ds_stage_copy(P.inter, P.gu, xsp, corr_f);  // the gate|up epilogue stored silu(g) * u
    else
      ds_stage_swiglu(P.inter, P.gu, xsp, corr_f);
    staged();
    run_projection(mb + 3);  // h += W_down silu(g) * u
  }
  ds_grid_barrier(P.bar, bar_base, err0, P.stamps, nbar, fill_rings);
  ds_stage_norm(P, P.hidden, P.norms[2 * P.layers], nullptr, xsp, redp, corr_f);
  staged();
  run_projection(nmats - 1);  // logits = W_head rmsnorm(h)

  // every unit issued was consumed (or, after a failed wait, drained); nothing is in flight
  if (P.stamps) {
    __syncthreads();
    if (threadIdx.x == 0) P.stamps[(size_t)gridDim.x + blockIdx.x] = globaltimer_ns();  // slot 1: end
  }
}

// ===================================================================== host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn ds_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

// Host object behind w4a16_decode_plan: the device tables and the step's scratch.
struct DecodePlan {
  int device = 0;
  int grid = 0;
  int smem = 0;
  void* tables = nullptr;   // [DsMat x nmats][tensor maps x 2 nmats][norm pointers]
  void* scratch = nullptr;  // h, qkv, attn, gu, partials, counters, barrier (zero-filled)
  unsigned long long* stamps = nullptr;  // timeline of the last step, when enabled
  size_t nstamps = 0;
  DsParams params = {};
  int layers = 0, kv_heads = 0, max_len = 0, hidden = 0, vocab = 0;
};

// Barriers of one step: four per layer after the first, five for every other layer, and
// the one before the head (layers * 5 in all).
int decode_step_barriers(int layers) { return layers * 5; }

int decode_plan_create(const w4a16_llama_desc* d, DecodePlan** out) {
  *out = nullptr;
  if (!d) {
    set_error("null model description");
    return W4A16_ERR_NULL;
  }
  const int L = d->layers, H = d->hidden, I = d->intermediate, NH = d->heads, KV = d->kv_heads;
  if (L < 1 || H <= 0 || I <= 0 || NH <= 0 || KV <= 0 || NH % KV != 0 || NH / KV > kDsWarps ||
      d->head_dim != kHeadDim || d->vocab <= 0 || d->max_len <= 0 || H % kWinCols || I % kWinCols ||
      (NH * kHeadDim) % kWinCols || H > kMaxNormK || I > kMaxStageK || NH * kHeadDim > kMaxStageK) {
    set_error("unsupported decode-step shape: layers %d hidden %d intermediate %d heads %d kv_heads %d "
              "head_dim %d vocab %d max_len %d (head_dim 64; hidden, intermediate and heads*64 multiples of "
              "1024, hidden <= %d, the others <= %d; heads / kv_heads <= %d)",
              L, H, I, NH, KV, d->head_dim, d->vocab, d->max_len, kMaxNormK, kMaxStageK, kDsWarps);
    return W4A16_ERR_SHAPE;
  }
  if (d->gate_up_interleaved != 0 && d->gate_up_interleaved != 8) {
    set_error("gate_up_interleaved must be 0 (gate | up) or 8 (blocks of 8 rows), got %d", d->gate_up_interleaved);
    return W4A16_ERR_SHAPE;
  }
  if (!d->qkv || !d->o || !d->gate_up || !d->down || !d->norm_attn || !d->norm_mlp || !d->norm_final ||
      !d->embed || !d->rope_cos || !d->rope_sin || !d->lm_head.packed || !d->lm_head.scale) {
    set_error("null pointer in the model description");
    return W4A16_ERR_NULL;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  int sms = 0, smem_optin = 0;
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) {
    set_error("device query: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  const int kmax = H > I ? (H > NH * kHeadDim ? H : NH * kHeadDim) : (I > NH * kHeadDim ? I : NH * kHeadDim);
  // x area: [the QKV phase's vector (2 hidden bytes) | the attention state: rotated queries,
  // new key and value, per-warp slice partials][attention rows: K | V of 32 positions];
  // the other phases use it whole for their vectors
  const int attn_state = (NH / KV + 2) * kHeadDim * 4 + kDsWarps * (kHeadDim + 2) * 4;
  const int kv_off = (int)align_up((size_t)(2 * H > attn_state ? 2 * H : attn_state), 128);
  const int kv_end = kv_off + 2 * kAttnSpan * kHeadDim * 2;
  const int xbytes = (int)align_up((size_t)(kmax * 2 > kv_end ? kmax * 2 : kv_end), 128);
  // [x | attention state][128 B scratch][corrections: kmax / 128 floats][local partials]
  // [projection table]
  const int lpart_off = xbytes + 128 + (int)align_up((size_t)(kmax / 128) * 4, 128);
  const int table_off = lpart_off + kLocalMaxWindows * kMmaRows * 4;
  static_assert((kLocalMaxWindows * kMmaRows * 4) % 128 == 0, "table offset alignment");
  const int smem = DsPlanLayout::kXOff + table_off + (4 * L + 1) * (int)sizeof(DsMat) + 1024;
  if (smem > smem_optin) {
    set_error("decode step needs %d bytes of shared memory, the device allows %d", smem, smem_optin);
    return W4A16_ERR_SHAPE;
  }
  e = cudaFuncSetAttribute(k_decode_step, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  int per_sm = 0;
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_step, kDsThreads, smem);
  if (e != cudaSuccess || per_sm < 1) {
    set_error("decode step kernel cannot be resident: %s (%d per SM)", cudaGetErrorString(e), per_sm);
    return W4A16_ERR_CUDA;
  }
  const int grid = sms;  // one CTA per SM; the cooperative launch checks co-residency
  const int W = grid * kDsWarps;

  // projections: per layer qkv, o, gate|up, down; then the head
  const int nmats = 4 * L + 1;
  std::vector<w4a16_g128_weight> ws(nmats);
  std::vector<int> rows(nmats), cols(nmats);
  const int qkv_rows = (NH + 2 * KV) * kHeadDim;
  for (int l = 0; l < L; ++l) {
    ws[4 * l + 0] = d->qkv[l];     rows[4 * l + 0] = qkv_rows;  cols[4 * l + 0] = H;
    ws[4 * l + 1] = d->o[l];       rows[4 * l + 1] = H;         cols[4 * l + 1] = NH * kHeadDim;
    ws[4 * l + 2] = d->gate_up[l]; rows[4 * l + 2] = 2 * I;     cols[4 * l + 2] = H;
    ws[4 * l + 3] = d->down[l];    rows[4 * l + 3] = H;         cols[4 * l + 3] = I;
  }
  ws[nmats - 1] = d->lm_head;
  rows[nmats - 1] = d->vocab;
  cols[nmats - 1] = H;
  for (int i = 0; i < nmats; ++i) {
    if (!ws[i].packed || !ws[i].scale || (reinterpret_cast<uintptr_t>(ws[i].packed) & 15) ||
        (reinterpret_cast<uintptr_t>(ws[i].scale) & 15)) {
      set_error("projection %d: weights and scales must be non-null and 16-byte aligned", i);
      return ws[i].packed && ws[i].scale ? W4A16_ERR_ALIGN : W4A16_ERR_NULL;
    }
  }
  for (int l = 0; l < L; ++l)
    if (!d->norm_attn[l] || !d->norm_mlp[l]) {
      set_error("layer %d: null norm weight", l);
      return W4A16_ERR_NULL;
    }

  // work split: projections whose CTA share fits the warps' rings at once run CTA-local
  // (windows added in shared memory), the others (the head) by whole tiles per warp; the
  // rotation moves each projection's extra work onto other CTAs / warps than the last one's
  std::vector<DsMat> mats(nmats);
  long long cum_tiles = 0, cum_units = 0, cum_windows = 0;
  for (int i = 0; i < nmats; ++i) {
    DsMat& m = mats[i];
    m.rows = rows[i];
    m.cols = cols[i];
    m.ntiles = (rows[i] + kMmaRows - 1) / kMmaRows;
    m.nwin = (cols[i] + kWinCols - 1) / kWinCols;
    const long long per_cta = ((long long)m.ntiles + grid - 1) / grid;
    m.mode = per_cta * m.nwin <= kLocalMaxWindows ? kModeLocal : kModeTile;
    m.woff = 0;
    m.tq = m.ntiles / grid;
    m.tr = m.ntiles % grid;
    if (m.mode == kModeLocal) {
      m.off = (int)(cum_tiles % grid);
      m.woff = (int)(cum_windows % kDsWarps);
      cum_tiles += m.ntiles;
      cum_windows += per_cta * m.nwin;
    } else {
      m.off = (int)(cum_units % W);
      cum_units += m.ntiles;
    }
  }
  const int splits = (d->max_len + kAttnSpan - 1) / kAttnSpan;  // attention chunks per kv head
  size_t off = 0;
  const size_t o_h = off;      off = align_up(off + (size_t)H * 4, 256);
  const size_t o_qkv = off;    off = align_up(off + (size_t)qkv_rows * 2, 256);
  const size_t o_attn = off;   off = align_up(off + (size_t)NH * kHeadDim * 2, 256);
  const size_t o_gu = off;     off = align_up(off + (size_t)2 * I * 2, 256);
  const size_t o_apart = off;  off = align_up(off + (size_t)NH * splits * (kHeadDim + 2) * 4, 256);
  const size_t o_acnt = off;   off = align_up(off + (size_t)KV * 4, 256);
  const size_t o_bar = off;    off = align_up(off + 8, 256);
  const size_t scratch_bytes = off;

  // tables: DsMat array, tensor maps (64-byte aligned), norm pointers
  const size_t t_mats = 0;
  const size_t t_maps = align_up(sizeof(DsMat) * nmats, 128);
  const size_t t_norms = align_up(t_maps + sizeof(CUtensorMap) * 2 * nmats, 128);
  const size_t table_bytes = t_norms + sizeof(float*) * (2 * L + 1);

  EncodeTiledFn enc = ds_encode_fn();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled entry point unavailable");
    return W4A16_ERR_CUDA;
  }
  std::vector<CUtensorMap> maps(2 * nmats);
  for (int i = 0; i < nmats; ++i) {
    const cuuint64_t dims[3] = {128, (cuuint64_t)(cols[i] / kSlabCols), (cuuint64_t)rows[i]};
    const cuuint64_t strides[2] = {128, (cuuint64_t)(cols[i] / 2)};
    const cuuint32_t box[3] = {128, (cuuint32_t)kDsSlabs, (cuuint32_t)kMmaRows};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(&maps[2 * i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(ws[i].packed), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS) {
      const cuuint64_t sd[2] = {(cuuint64_t)(cols[i] / 128), (cuuint64_t)rows[i]};
      const cuuint64_t ss[1] = {(cuuint64_t)(cols[i] / 128) * 4};
      const cuuint32_t sbox[2] = {(cuuint32_t)DsL::kGroups, (cuuint32_t)kMmaRows};
      const cuuint32_t se[2] = {1, 1};
      r = enc(&maps[2 * i + 1], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ws[i].scale), sd, ss,
              sbox, se, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled failed for projection %d: %d", i, (int)r);
      return W4A16_ERR_CUDA;
    }
  }

  DecodePlan* plan = new DecodePlan();
  plan->device = dev;
  plan->grid = grid;
  plan->smem = smem;
  plan->layers = L;
  plan->kv_heads = KV;
  plan->max_len = d->max_len;
  plan->hidden = H;
  plan->vocab = d->vocab;
  e = cudaMalloc(&plan->tables, table_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&plan->scratch, scratch_bytes);
  if (e == cudaSuccess) e = cudaMemset(plan->scratch, 0, scratch_bytes);
  uint8_t* tb = static_cast<uint8_t*>(plan->tables);
  uint8_t* sc = static_cast<uint8_t*>(plan->scratch);
  if (e == cudaSuccess) {
    const CUtensorMap* dmaps = reinterpret_cast<const CUtensorMap*>(tb + t_maps);
    for (int i = 0; i < nmats; ++i) {
      mats[i].wmap = dmaps + 2 * i;
      mats[i].smap = dmaps + 2 * i + 1;
      const int kind = i == nmats - 1 ? kOutFloat
                       : (i % 4 == 1 || i % 4 == 3) ? kOutResidual
                       : (i % 4 == 2 && d->gate_up_interleaved) ? kOutSwiGlu : kOutHalf;
      mats[i].out_kind = kind;
      mats[i].out = i == nmats - 1 ? nullptr  // the logits buffer is a step argument
                    : kind == kOutResidual ? static_cast<void*>(sc + o_h)
                    : i % 4 == 0 ? static_cast<void*>(sc + o_qkv) : static_cast<void*>(sc + o_gu);
    }
    std::vector<const float*> norms(2 * L + 1);
    for (int l = 0; l < L; ++l) {
      norms[2 * l] = d->norm_attn[l];
      norms[2 * l + 1] = d->norm_mlp[l];
    }
    norms[2 * L] = d->norm_final;
    e = cudaMemcpy(tb + t_mats, mats.data(), sizeof(DsMat) * nmats, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
      e = cudaMemcpy(tb + t_maps, maps.data(), sizeof(CUtensorMap) * 2 * nmats, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
      e = cudaMemcpy(tb + t_norms, norms.data(), sizeof(float*) * (2 * L + 1), cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) {
    set_error("decode plan: %s", cudaGetErrorString(e));
    if (plan->tables) cudaFree(plan->tables);
    if (plan->scratch) cudaFree(plan->scratch);
    delete plan;
    return W4A16_ERR_CUDA;
  }
  DsParams& p = plan->params;
  p.mats = reinterpret_cast<const DsMat*>(tb + t_mats);
  p.norms = reinterpret_cast<const float* const*>(tb + t_norms);
  p.embed = static_cast<const __half*>(d->embed);
  p.cos_t = d->rope_cos;
  p.sin_t = d->rope_sin;
  p.h = reinterpret_cast<float*>(sc + o_h);
  p.qkv = reinterpret_cast<__half*>(sc + o_qkv);
  p.attn = reinterpret_cast<__half*>(sc + o_attn);
  p.gu = reinterpret_cast<__half*>(sc + o_gu);
  p.attn_part = reinterpret_cast<float*>(sc + o_apart);
  p.attn_cnt = reinterpret_cast<unsigned*>(sc + o_acnt);
  p.bar = reinterpret_cast<unsigned long long*>(sc + o_bar);
  p.layers = L;
  p.hidden = H;
  p.inter = I;
  p.heads = NH;
  p.kv_heads = KV;
  p.max_len = d->max_len;
  p.splits = splits;
  p.nmats = nmats;
  p.vocab = d->vocab;
  p.gu_interleaved = d->gate_up_interleaved ? 1 : 0;
  p.kv_off = kv_off;
  p.lpart_off = lpart_off;
  p.table_off = table_off;
  p.xbytes = xbytes;
  p.eps = d->eps;
  *out = plan;
  return W4A16_OK;
}

int decode_plan_timeline(DecodePlan* plan, int enable, unsigned long long* host, size_t capacity,
                         size_t* count, cudaStream_t stream) {
  const size_t n = (size_t)3 * (decode_step_barriers(plan->layers) + 1) * plan->grid;
  if (count) *count = n;
  if (enable && !plan->stamps) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, n * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(p, 0, n * sizeof(unsigned long long));
    if (e != cudaSuccess) {
      set_error("timeline buffer: %s", cudaGetErrorString(e));
      return W4A16_ERR_CUDA;
    }
    plan->stamps = static_cast<unsigned long long*>(p);
    plan->nstamps = n;
  }
  if (host && plan->stamps) {
    if (capacity < n) {
      set_error("timeline needs %zu entries, got %zu", n, capacity);
      return W4A16_ERR_SHAPE;
    }
    cudaError_t e = cudaMemcpyAsync(host, plan->stamps, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                                    stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
      set_error("reading the timeline: %s", cudaGetErrorString(e));
      return W4A16_ERR_CUDA;
    }
  }
  if (!enable && plan->stamps) {
    cudaError_t e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess) e = cudaFree(plan->stamps);
    plan->stamps = nullptr;
    plan->nstamps = 0;
    if (e != cudaSuccess) {
      set_error("freeing the timeline: %s", cudaGetErrorString(e));
      return W4A16_ERR_CUDA;
    }
  }
  plan->params.stamps = plan->stamps;
  return W4A16_OK;
}

int decode_plan_destroy(DecodePlan* plan) {
  if (!plan) return W4A16_OK;
  if (plan->stamps) cudaFree(plan->stamps);
  cudaError_t e1 = plan->tables ? cudaFree(plan->tables) : cudaSuccess;
  cudaError_t e2 = plan->scratch ? cudaFree(plan->scratch) : cudaSuccess;
  delete plan;
  if (e1 != cudaSuccess || e2 != cudaSuccess) {
    set_error("freeing the decode plan: %s", cudaGetErrorString(e1 != cudaSuccess ? e1 : e2));
    return W4A16_ERR_CUDA;
  }
  return W4A16_OK;
}

int decode_step_launch(DecodePlan* plan, const long long* token, const long long* pos, void* k_cache,
                       void* v_cache, float* logits, cudaStream_t stream) {
  DsParams p = plan->params;
  p.token = token;
  p.pos = pos;
  p.k_cache = static_cast<__half*>(k_cache);
  p.v_cache = static_cast<__half*>(v_cache);
  p.logits = logits;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan->grid);
  cfg.blockDim = dim3(kDsThreads);
  cfg.dynamicSmemBytes = plan->smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_decode_step, p);
  (void)cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("k_decode_step launch failed: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  return W4A16_OK;
}

int read_decode_step_error(int* code, cudaStream_t stream) {
  int h = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_ds_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess && h != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_ds_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  }
  if (e != cudaSuccess) {
    set_error("reading the decode-step error word: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  *code = h;
  return W4A16_OK;
}

}  // namespace w4a16
