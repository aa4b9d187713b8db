// W4A16 GEMV kernels for B200 (sm_100a).
//
// Main path (k_gemv_tma): every warp owns a private ring of shared-memory stages
// that TMA (cp.async.bulk.tensor, 128-byte swizzle) fills with 16-row x 1024-column
// tiles of packed int4 weights (and, for group-128, the matching scale tile).  The
// warp decodes each packed word to f16x2 codes in registers (decode_word: shift +
// 4 lop3 + 4 f16x2 ops, exact) and feeds them as the A operand of
// mma.sync.m16n8k16 with the activation as the B operand, so products are exact and
// accumulation is fp32 in the tensor core.  Columns of B carry up to 8 (16 with two
// MMAs) activation rows: batch 1..16 costs the same weight traffic as batch 1.
// Group-128 partial sums are scaled in fp32 once per group; per-row sums once per
// row.  Items (16 rows x a K range) are spread warp-major over a persistent grid of
// one CTA per SM; layers with few rows split K across warps and the last warp to
// finish a tile reduces the partials in a fixed order (deterministic).
//
// Reference counterparts: k_marlin (kernels/w4a16_kernels.cu:100-114) and
// k_marlin_g128 (:121-138) compute the same sums with one warp per row, 4-byte
// weight loads and CUDA-core FMAs.
//
// Fallback (k_gemv_generic): one warp per row, CUDA-core fp32 FMAs, any cols % 8,
// any alignment the C ABI accepts.  Used when the TMA constraints do not hold.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <type_traits>

#include "w4a16_device.cuh"
#include "w4a16_internal.h"

#ifndef W4A16_TMA_WARPS
#define W4A16_TMA_WARPS 8
#endif
#ifndef W4A16_TMA_STAGES
#define W4A16_TMA_STAGES 3
#endif
#ifndef W4A16_TMA_SLABS
#define W4A16_TMA_SLABS 4
#endif

namespace w4a16 {

// First error code raised by a kernel on this device since the last read.
__device__ int g_device_error = 0;

enum DeviceErrorCode : int {
  kDevErrStageTimeout = 1,  // a TMA stage did not land within the wait limit
};

constexpr uint64_t kStageWaitLimitNs = 2000000000ull;  // 2 s; a stage normally lands in us
constexpr uint64_t kDrainWaitLimitNs = 100000000ull;   // 0.1 s per outstanding stage

__device__ __forceinline__ void record_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

constexpr int kTileRows = 16;     // rows per item (the M of one m16n8k16)
constexpr int kSlabCols = 256;    // columns per 128-byte TMA box row
constexpr int kSlabBytes = kTileRows * 128;
constexpr int kMaxBatchPerPass = 16;
// Split-K workspace layout: [tile counters: kMaxSplitTiles x u32][fp32 partials].
// The counter region has a fixed size so that calls of different shapes sharing one
// workspace never see another call's partials where they expect zeroed counters.
constexpr int kMaxSplitTiles = 4096;
constexpr size_t kCounterBytes = (size_t)kMaxSplitTiles * 4;

struct TmaParams {
  const void* scale_rows;  // per-row scale [N] (group 0)
  const __half* x;         // [M][K]
  void* y;                 // [M][N]
  const float* bias;       // [N] or null
  float* partial;          // [nsplit][M][N] when nsplit > 1
  unsigned* counters;      // [ntiles] when nsplit > 1
  int M, N, K;
  int ntiles, nsplit, stages_per_split, nstages, n_items;
};

template <int SLABS, int GS, typename ST>
struct StageLayout {
  static constexpr int kWBytes = SLABS * kSlabBytes;
  static constexpr int kGroups = SLABS * 2;  // 128-column groups per stage
  static constexpr int kSBytes = GS ? kTileRows * kGroups * (int)sizeof(ST) : 0;
  static constexpr int kBytes = (kWBytes + kSBytes + 1023) / 1024 * 1024;
};

template <int NB>
struct BatchCfg {
  static constexpr int kHalves = NB > 8 ? 2 : 1;  // n8 MMAs per A fragment
};

// Activation fragment for column block h: row n = h*8 + g of X (all rows = X[0]
// when NB == 1, so every B column holds the single vector).
template <int NB>
__device__ __forceinline__ uint4 load_x(const __half* x, int K, int M, int g, int h, int col) {
  if (NB == 1) return ldg128(x + col);
  const int n = h * 8 + g;
  if (n < M) return ldg128(x + (size_t)n * K + col);
  return make_uint4(0u, 0u, 0u, 0u);
}

template <int PACK, int GS, typename ST, int NB, typename OT, int WARPS, int STAGES, int SLABS>
__global__ void __launch_bounds__(WARPS * 32, 1)
    k_gemv_tma(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
               const TmaParams p) {
  using L = StageLayout<SLABS, GS, ST>;
  constexpr int NH = BatchCfg<NB>::kHalves;
  static_assert(!GS || (L::kGroups * sizeof(ST)) % 16 == 0, "scale box row must be 16-byte multiple");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;  // MMA group id: rows g and g+8 of the tile
  const int t = lane & 3;   // thread in group: 32-column chunk t of each 128-column group

  const int gw = warp * gridDim.x + blockIdx.x;  // warp-major: items spread over all SMs
  if (gw >= p.n_items) return;
  const int total_warps = gridDim.x * WARPS;

  const uint32_t ring = base + (uint32_t)(warp * STAGES * L::kBytes);
  const uint32_t bar0 = base + (uint32_t)(WARPS * STAGES * L::kBytes + warp * STAGES * 8);

  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(bar0 + 8 * s, 1);
    mbar_fence_init();
    tma_prefetch_desc(&wmap);
    if (GS) tma_prefetch_desc(&smap);
  }
  __syncwarp();
  const uint64_t policy = l2_policy_evict_first();
  const int kslabs = p.K / kSlabCols;

  // Producer cursor (kept identical in every lane; lane 0 issues).
  int p_item = gw;
  int p_stage = (p_item % p.nsplit) * p.stages_per_split;
  int p_end = min(p_stage + p.stages_per_split, p.nstages);
  uint32_t issued = 0;

  auto issue_one = [&]() {
    if (p_item >= p.n_items) return;
    const uint32_t slot = issued % STAGES;
    if (lane == 0) {
      const int tile = p_item / p.nsplit;
      const int nslab = min(SLABS, kslabs - p_stage * SLABS);
      const uint32_t dst = ring + slot * L::kBytes;
      const uint32_t bar = bar0 + 8 * slot;
      mbar_arrive_expect_tx(bar, (uint32_t)(nslab * kSlabBytes + L::kSBytes));
      for (int sl = 0; sl < nslab; ++sl)
        tma_load_2d(dst + sl * kSlabBytes, &wmap, (p_stage * SLABS + sl) * 128, tile * kTileRows,
                    bar, policy);
      if (GS) tma_load_2d(dst + L::kWBytes, &smap, p_stage * L::kGroups, tile * kTileRows, bar, policy);
    }
    ++issued;
    if (++p_stage == p_end) {
      p_item += total_warps;
      p_stage = (p_item % p.nsplit) * p.stages_per_split;
      p_end = min(p_stage + p.stages_per_split, p.nstages);
    }
  };

#pragma unroll 1
  for (int s = 0; s < STAGES; ++s) issue_one();

  uint32_t consumed = 0;
#pragma unroll 1
  for (int item = gw; item < p.n_items; item += total_warps) {
    const int tile = item / p.nsplit;
    const int split = item % p.nsplit;
    const int st_begin = split * p.stages_per_split;
    const int st_end = min(st_begin + p.stages_per_split, p.nstages);
    const int r0 = tile * kTileRows + g;
    const int r1 = r0 + 8;

    // Per-row scales are needed only in the epilogue: fetch them now.
    float srow0 = 1.f, srow1 = 1.f;
    if (!GS) {
      const ST* sr = static_cast<const ST*>(p.scale_rows);
      if (r0 < p.N) srow0 = to_f32<ST>(__ldg(sr + r0));
      if (r1 < p.N) srow1 = to_f32<ST>(__ldg(sr + r1));
    }

    float tot[NH][4];
    float acc[2][NH][4];
#pragma unroll
    for (int h = 0; h < NH; ++h)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        tot[h][i] = 0.f;
        acc[0][h][i] = 0.f;
        acc[1][h][i] = 0.f;
      }

#pragma unroll 1
    for (int stage = st_begin; stage < st_end; ++stage) {
      const uint32_t slot = consumed % STAGES;
      const uint32_t parity = (consumed / STAGES) & 1u;
      if (!mbar_wait_bounded(bar0 + 8 * slot, parity, kStageWaitLimitNs)) {
        record_device_error(kDevErrStageTimeout);
        for (uint32_t s = consumed + 1; s < issued; ++s)
          mbar_wait_bounded(bar0 + 8 * (s % STAGES), (s / STAGES) & 1u, kDrainWaitLimitNs);
        return;
      }
      const uint32_t sbase = ring + slot * L::kBytes;
      const int nslab = min(SLABS, kslabs - stage * SLABS);

#pragma unroll
      for (int sl = 0; sl < SLABS; ++sl) {
        if (sl < nslab) {
          const uint32_t slab = sbase + sl * kSlabBytes;
          const int kcol = (stage * SLABS + sl) * kSlabCols;
          // 128-byte swizzle: 16-byte chunk c of smem row r sits at chunk c ^ (r & 7).
          uint4 wa[2], wb[2];
#pragma unroll
          for (int gh = 0; gh < 2; ++gh) {
            const uint32_t c = (uint32_t)((gh * 4 + t) ^ g);
            wa[gh] = lds128(slab + g * 128 + c * 16);
            wb[gh] = lds128(slab + (g + 8) * 128 + c * 16);
          }
          if (GS) {
#pragma unroll
            for (int gh = 0; gh < 2; ++gh)
#pragma unroll
              for (int h = 0; h < NH; ++h)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[gh][h][i] = 0.f;
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int gh = 0; gh < 2; ++gh) {
              const uint32_t word_a = j == 0 ? wa[gh].x : j == 1 ? wa[gh].y : j == 2 ? wa[gh].z : wa[gh].w;
              const uint32_t word_b = j == 0 ? wb[gh].x : j == 1 ? wb[gh].y : j == 2 ? wb[gh].z : wb[gh].w;
              uint32_t A[4], B[4];
              decode_word(word_a, A);
              decode_word(word_b, B);
              const int col = kcol + gh * 128 + 32 * t + 8 * j;
#pragma unroll
              for (int h = 0; h < NH; ++h) {
                uint4 xv = load_x<NB>(p.x, p.K, p.M, g, h, col);
                if (PACK == W4A16_PACK_SIMPLE) xv = simple_order(xv);
                mma_16816(acc[gh][h], A[0], B[0], A[1], B[1], xv.x, xv.y);
                mma_16816(acc[gh][h], A[2], B[2], A[3], B[3], xv.z, xv.w);
              }
            }
          }
          if (GS) {
            const uint32_t sb = sbase + L::kWBytes;
#pragma unroll
            for (int gh = 0; gh < 2; ++gh) {
              const int grp = sl * 2 + gh;
              float s0, s1;
              if (sizeof(ST) == 4) {
                s0 = lds_f32(sb + (g * L::kGroups + grp) * 4);
                s1 = lds_f32(sb + ((g + 8) * L::kGroups + grp) * 4);
              } else {
                s0 = __half2float(__ushort_as_half(lds_u16(sb + (g * L::kGroups + grp) * 2)));
                s1 = __half2float(__ushort_as_half(lds_u16(sb + ((g + 8) * L::kGroups + grp) * 2)));
              }
#pragma unroll
              for (int h = 0; h < NH; ++h) {
                tot[h][0] = fmaf(s0, acc[gh][h][0], tot[h][0]);
                tot[h][1] = fmaf(s0, acc[gh][h][1], tot[h][1]);
                tot[h][2] = fmaf(s1, acc[gh][h][2], tot[h][2]);
                tot[h][3] = fmaf(s1, acc[gh][h][3], tot[h][3]);
              }
            }
          }
        }
      }
      __syncwarp();  // every lane has read the slot before it is refilled
      ++consumed;
      issue_one();
    }

    if (!GS) {
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        tot[h][0] = (acc[0][h][0] + acc[1][h][0]) * srow0;
        tot[h][1] = (acc[0][h][1] + acc[1][h][1]) * srow0;
        tot[h][2] = (acc[0][h][2] + acc[1][h][2]) * srow1;
        tot[h][3] = (acc[0][h][3] + acc[1][h][3]) * srow1;
      }
    }

    // Fragment (h, i): row r0 (i < 2) or r1, batch column n = h*8 + 2t + (i & 1).
    if (p.nsplit == 1) {
#pragma unroll
      for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = i < 2 ? r0 : r1;
          const int n = h * 8 + 2 * t + (i & 1);
          const bool ok = NB == 1 ? (t == 0 && (i & 1) == 0) : (n < p.M);
          if (ok && r < p.N) {
            float v = tot[h][i];
            if (p.bias) v += __ldg(p.bias + r);
            static_cast<OT*>(p.y)[(size_t)n * p.N + r] = from_f32<OT>(v);
          }
        }
    } else {
#pragma unroll
      for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = i < 2 ? r0 : r1;
          const int n = h * 8 + 2 * t + (i & 1);
          const bool ok = NB == 1 ? (t == 0 && (i & 1) == 0) : (n < p.M);
          if (ok && r < p.N) p.partial[((size_t)split * p.M + n) * p.N + r] = tot[h][i];
        }
      __threadfence();
      __syncwarp();
      unsigned prev = 0;
      if (lane == 0) prev = atomicAdd(p.counters + tile, 1u);
      prev = __shfl_sync(0xffffffffu, prev, 0);
      if (prev == (unsigned)(p.nsplit - 1)) {
        __threadfence();
#pragma unroll
        for (int h = 0; h < NH; ++h)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = i < 2 ? r0 : r1;
            const int n = h * 8 + 2 * t + (i & 1);
            const bool ok = NB == 1 ? (t == 0 && (i & 1) == 0) : (n < p.M);
            if (ok && r < p.N) {
              float v = 0.f;
              for (int s = 0; s < p.nsplit; ++s)
                v += __ldcg(p.partial + ((size_t)s * p.M + n) * p.N + r);
              if (p.bias) v += __ldg(p.bias + r);
              static_cast<OT*>(p.y)[(size_t)n * p.N + r] = from_f32<OT>(v);
            }
          }
        __syncwarp();
        if (lane == 0) p.counters[tile] = 0u;  // leave the workspace zeroed
      }
    }
  }
}

// ------------------------------------------------------------ generic fallback

template <int PACK, int GS, typename ST, typename OT>
__global__ void __launch_bounds__(256)
    k_gemv_generic(const uint8_t* __restrict__ packed, const ST* __restrict__ scale,
                   const __half* __restrict__ x, OT* __restrict__ y, const float* __restrict__ bias,
                   int M, int N, int K) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= N) return;
  const uint8_t* wrow = packed + (size_t)row * (K >> 1);
  const int words = K >> 3;
  const int ngroups = GS ? K / (GS ? GS : 1) : 1;
  float acc[kMaxBatchPerPass];
#pragma unroll
  for (int m = 0; m < kMaxBatchPerPass; ++m) acc[m] = 0.f;

  for (int w = lane; w < words; w += 32) {
    const uint32_t word = __ldg(reinterpret_cast<const uint32_t*>(wrow) + w);
    uint32_t o[4];
    decode_word(word, o);
    float wf[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&o[i]));
      wf[2 * i] = f.x;
      wf[2 * i + 1] = f.y;
    }
    const float s = GS ? to_f32<ST>(__ldg(scale + (size_t)row * ngroups + (w * 8) / (GS ? GS : 1))) : 1.f;
#pragma unroll
    for (int m = 0; m < kMaxBatchPerPass; ++m) {
      if (m < M) {
        uint4 xv = ldg128(x + (size_t)m * K + (size_t)w * 8);
        if (PACK == W4A16_PACK_SIMPLE) xv = simple_order(xv);
        const uint32_t xr[4] = {xv.x, xv.y, xv.z, xv.w};
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 xf = __half22float2(*reinterpret_cast<const __half2*>(&xr[i]));
          d = fmaf(wf[2 * i], xf.x, d);
          d = fmaf(wf[2 * i + 1], xf.y, d);
        }
        acc[m] = GS ? fmaf(s, d, acc[m]) : acc[m] + d;
      }
    }
  }
#pragma unroll
  for (int m = 0; m < kMaxBatchPerPass; ++m) {
    if (m < M) {
      float v = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[m] = v;
    }
  }
  if (lane == 0) {
    const float srow = GS ? 1.f : to_f32<ST>(__ldg(scale + row));
    const float b = bias ? __ldg(bias + row) : 0.f;
    for (int m = 0; m < M; ++m) y[(size_t)m * N + row] = from_f32<OT>(acc[m] * srow + b);
  }
}

// =================================================================== host side

namespace {

thread_local char t_last_error[512] = "";

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int sms = 0;
  int smem_optin = 0;
};

int current_device_info(DeviceInfo* out, int* dev_out) {
  static std::mutex mu;
  static DeviceInfo cache[kMaxDevices];
  static bool have[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("cudaGetDevice: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("device index %d out of range", dev);
    return W4A16_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!have[dev]) {
    DeviceInfo d;
    e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) {
      set_error("cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
      return W4A16_ERR_CUDA;
    }
    cache[dev] = d;
    have[dev] = true;
  }
  *out = cache[dev];
  if (dev_out) *dev_out = dev;
  return W4A16_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s launch failed: %s", what, cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  return W4A16_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

constexpr int kWarps = W4A16_TMA_WARPS;
constexpr int kStages = W4A16_TMA_STAGES;
constexpr int kSlabs = W4A16_TMA_SLABS;
constexpr int kStageCols = kSlabs * kSlabCols;

template <int GS, typename ST>
constexpr int tma_smem_bytes() {
  return kWarps * kStages * StageLayout<kSlabs, GS, ST>::kBytes + kWarps * kStages * 8 + 1024;
}

// Split count for a problem: enough items to occupy every warp slot when the
// layer has few row tiles.
int choose_split(int ntiles, int nstages, int slots) {
  if (ntiles * 2 > slots || nstages < 2) return 1;
  int s = (slots + ntiles - 1) / ntiles;
  return s < nstages ? s : nstages;
}

template <int PACK, int GS, typename ST, int NB, typename OT>
int launch_tma(const GemvProblem& p, const __half* x, int M, void* y, int nsplit, int stages_per_split,
               const DeviceInfo& di, int dev) {
  auto kernel = k_gemv_tma<PACK, GS, ST, NB, OT, kWarps, kStages, kSlabs>;
  constexpr int smem = tma_smem_bytes<GS, ST>();
  static std::atomic<uint64_t> configured{0};
  const uint64_t bit = 1ull << dev;
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(%d bytes): %s", smem, cudaGetErrorString(e));
      return W4A16_ERR_CUDA;
    }
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }

  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled entry point unavailable");
    return W4A16_ERR_CUDA;
  }
  CUtensorMap wmap, smap;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)(p.K / 2), (cuuint64_t)p.N};
    const cuuint64_t strides[1] = {(cuuint64_t)(p.K / 2)};
    const cuuint32_t box[2] = {128, kTileRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(p.packed),
                           dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled(weights) failed: %d", (int)r);
      return W4A16_ERR_CUDA;
    }
  }
  if constexpr (GS != 0) {
    const int ng = p.K / GS;
    const cuuint64_t dims[2] = {(cuuint64_t)ng, (cuuint64_t)p.N};
    const cuuint64_t strides[1] = {(cuuint64_t)ng * sizeof(ST)};
    const cuuint32_t box[2] = {(cuuint32_t)StageLayout<kSlabs, GS, ST>::kGroups, kTileRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt =
        sizeof(ST) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const CUresult r = enc(&smap, dt, 2, const_cast<void*>(p.scale), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled(scales) failed: %d", (int)r);
      return W4A16_ERR_CUDA;
    }
  } else {
    smap = wmap;  // unused
  }

  TmaParams prm;
  prm.scale_rows = p.scale;
  prm.x = x;
  prm.y = y;
  prm.bias = p.bias;
  prm.M = M;
  prm.N = p.N;
  prm.K = p.K;
  prm.ntiles = (p.N + kTileRows - 1) / kTileRows;
  prm.nstages = (p.K + kStageCols - 1) / kStageCols;
  prm.nsplit = nsplit;
  prm.stages_per_split = stages_per_split;
  prm.n_items = prm.ntiles * nsplit;
  prm.partial = nullptr;
  prm.counters = nullptr;
  if (nsplit > 1) {
    uint8_t* ws = static_cast<uint8_t*>(p.workspace);
    prm.counters = reinterpret_cast<unsigned*>(ws);
    prm.partial = reinterpret_cast<float*>(ws + kCounterBytes);
  }
  int grid = (prm.n_items + kWarps - 1) / kWarps;
  if (prm.n_items >= di.sms) grid = di.sms;
  if (grid > di.sms) grid = di.sms;
  if (grid < 1) grid = 1;
  kernel<<<grid, kWarps * 32, smem, p.stream>>>(wmap, smap, prm);
  return check_launch("k_gemv_tma");
}

template <int PACK, int GS, typename ST, typename OT>
int launch_generic(const GemvProblem& p, const __half* x, int M, void* y) {
  const int threads = 256;
  const int rows_per_block = threads / 32;
  const int grid = (p.N + rows_per_block - 1) / rows_per_block;
  k_gemv_generic<PACK, GS, ST, OT><<<grid, threads, 0, p.stream>>>(
      p.packed, static_cast<const ST*>(p.scale), x, static_cast<OT*>(y), p.bias, M, p.N, p.K);
  return check_launch("k_gemv_generic");
}


template <int PACK, int GS, typename ST, typename OT>
int run_pass(const GemvProblem& p, const __half* x, int M, void* y, bool use_tma,
             const DeviceInfo& di, int dev) {
  // The simple packing (the reference's ladder kernels) only ever carries per-row
  // fp32 scales and fp32 outputs there; other combinations take the generic kernel.
  constexpr bool kTmaVariant =
      PACK == W4A16_PACK_INTERLEAVED ||
      (GS == 0 && std::is_same<ST, float>::value && std::is_same<OT, float>::value);
  if constexpr (!kTmaVariant) {
    (void)use_tma;
    (void)di;
    (void)dev;
    return launch_generic<PACK, GS, ST, OT>(p, x, M, y);
  } else {
  if (!use_tma) return launch_generic<PACK, GS, ST, OT>(p, x, M, y);
  const int ntiles = (p.N + kTileRows - 1) / kTileRows;
  const int nstages = (p.K + kStageCols - 1) / kStageCols;
  int nsplit = 1;
  if (p.split_k == 0) {
    nsplit = ntiles <= kMaxSplitTiles ? choose_split(ntiles, nstages, di.sms * kWarps) : 1;
  } else {
    nsplit = p.split_k < nstages ? p.split_k : nstages;
    if (ntiles > kMaxSplitTiles) nsplit = 1;
  }
  int sps = nstages;
  if (nsplit > 1) {
    sps = (nstages + nsplit - 1) / nsplit;
    nsplit = (nstages + sps - 1) / sps;
  }
  if (nsplit > 1) {
    const size_t need = kCounterBytes + (size_t)nsplit * M * p.N * 4;
    if (!p.workspace || p.workspace_bytes < need || !aligned(p.workspace, 256)) {
      if (p.split_k > 1) {
        set_error("split-K %d needs a 256-byte aligned workspace of %zu bytes (got %zu)",
                  p.split_k, need, p.workspace_bytes);
        return W4A16_ERR_WORKSPACE;
      }
      nsplit = 1;
      sps = nstages;
    }
  }
  if (M == 1) return launch_tma<PACK, GS, ST, 1, OT>(p, x, M, y, nsplit, sps, di, dev);
  if (M <= 8) return launch_tma<PACK, GS, ST, 8, OT>(p, x, M, y, nsplit, sps, di, dev);
  return launch_tma<PACK, GS, ST, 16, OT>(p, x, M, y, nsplit, sps, di, dev);
  }
}

template <int PACK, int GS, typename ST, typename OT>
int run_all(const GemvProblem& p, bool use_tma, const DeviceInfo& di, int dev) {
  const size_t osz = sizeof(OT);
  for (int m0 = 0; m0 < p.M; m0 += kMaxBatchPerPass) {
    const int mc = p.M - m0 < kMaxBatchPerPass ? p.M - m0 : kMaxBatchPerPass;
    const __half* x = static_cast<const __half*>(p.x) + (size_t)m0 * p.K;
    void* y = static_cast<uint8_t*>(p.y) + (size_t)m0 * p.N * osz;
    const int rc = run_pass<PACK, GS, ST, OT>(p, x, mc, y, use_tma, di, dev);
    if (rc != W4A16_OK) return rc;
  }
  return W4A16_OK;
}

}  // namespace

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

const char* last_error() { return t_last_error; }

size_t gemv_counter_bytes() { return kCounterBytes; }

size_t gemv_workspace_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int mc = M < kMaxBatchPerPass ? M : kMaxBatchPerPass;
  const size_t nstages = (size_t)(K + kStageCols - 1) / kStageCols;
  return kCounterBytes + nstages * (size_t)mc * N * 4;
}

int launch_gemv(const GemvProblem& p) {
  DeviceInfo di;
  int dev = 0;
  int rc = current_device_info(&di, &dev);
  if (rc != W4A16_OK) return rc;

  const size_t ssz = p.scale_dtype == W4A16_DTYPE_F32 ? 4 : 2;
  bool use_tma = (p.K % kSlabCols) == 0 && aligned(p.packed, 16) && aligned(p.x, 16);
  if (p.group) {
    const size_t row_bytes = (size_t)(p.K / p.group) * ssz;
    use_tma = use_tma && (row_bytes % 16) == 0 && aligned(p.scale, 16);
  }
  if (p.packing == W4A16_PACK_SIMPLE && (p.group || p.scale_dtype != W4A16_DTYPE_F32 ||
                                         p.out_dtype != W4A16_DTYPE_F32))
    use_tma = false;
  const int smem_need =
      p.group ? (p.scale_dtype == W4A16_DTYPE_F32 ? tma_smem_bytes<128, float>()
                                                  : tma_smem_bytes<128, __half>())
              : tma_smem_bytes<0, float>();
  if (smem_need > di.smem_optin) use_tma = false;

  const bool f32s = p.scale_dtype == W4A16_DTYPE_F32;
  const bool f32o = p.out_dtype == W4A16_DTYPE_F32;
  if (p.packing == W4A16_PACK_SIMPLE) {
    if (!p.group) {
      if (f32s)
        return f32o ? run_all<1, 0, float, float>(p, use_tma, di, dev)
                    : run_all<1, 0, float, __half>(p, use_tma, di, dev);
      return f32o ? run_all<1, 0, __half, float>(p, use_tma, di, dev)
                  : run_all<1, 0, __half, __half>(p, use_tma, di, dev);
    }
    if (f32s)
      return f32o ? run_all<1, 128, float, float>(p, use_tma, di, dev)
                  : run_all<1, 128, float, __half>(p, use_tma, di, dev);
    return f32o ? run_all<1, 128, __half, float>(p, use_tma, di, dev)
                : run_all<1, 128, __half, __half>(p, use_tma, di, dev);
  }
  if (!p.group) {
    if (f32s)
      return f32o ? run_all<0, 0, float, float>(p, use_tma, di, dev)
                  : run_all<0, 0, float, __half>(p, use_tma, di, dev);
    return f32o ? run_all<0, 0, __half, float>(p, use_tma, di, dev)
                : run_all<0, 0, __half, __half>(p, use_tma, di, dev);
  }
  if (f32s)
    return f32o ? run_all<0, 128, float, float>(p, use_tma, di, dev)
                : run_all<0, 128, float, __half>(p, use_tma, di, dev);
  return f32o ? run_all<0, 128, __half, float>(p, use_tma, di, dev)
              : run_all<0, 128, __half, __half>(p, use_tma, di, dev);
}

int read_device_error(int* code, cudaStream_t stream) {
  int h = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_device_error, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess && h != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice,
                                stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  }
  if (e != cudaSuccess) {
    set_error("reading the device error word: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  *code = h;
  return W4A16_OK;
}

}  // namespace w4a16
