// W4A16 GEMV kernels for B200 (sm_100a).
//
// Main path (k_gemv_tma): every warp owns a private ring of shared-memory stages
// that TMA (cp.async.bulk.tensor, 128-byte swizzle) fills with 16-row x 1024-column
// windows of packed int4 weights (one 3-D box per window) and, for group-128, the
// matching scale tile.  The warp decodes each packed word to f16x2 codes in
// registers (exact) and feeds them as the A operand of mma.sync.m16n8k16 with the
// activation as the B operand, so products are exact and accumulation is fp32 in the
// tensor core.  Columns of B carry up to 8 (16 with two MMAs) activation rows: batch
// 1..16 costs the same weight traffic as batch 1.  For one activation vector the
// decode leaves half of the nibbles biased by +72 (decode_word_fold, 7 instructions
// per word) and every 128-column group starts its accumulator at -72 * (sum of the
// activation over those columns); group-128 sums are scaled once per group in fp32,
// per-row sums once per row.
//
// One activation vector is staged in shared memory by the CTA, optionally computed
// on the way (RMSNorm of an fp32 vector, or SwiGLU of a gate|up vector: the decode
// step's prologues).  Launches may be chained (programmatic dependent launch): the
// weight copies start before the wait for the previous kernel.
//
// Work is split over (16-row tile, 1024-column window) units with a persistent grid
// of one CTA per SM: dynamic whole-tile pulls, stream-K ranges finished by the last
// contributor (partials added in warp order, deterministic), static whole tiles, or
// CTA-local ranges reduced in shared memory for small matrices (see Sched).  The
// fused all-gather (TP kernels only) writes each output row into every rank's buffer
// over NVLink and signals completion through flags in those buffers.
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
#include "w4a16_gemv_core.cuh"
#include "w4a16_internal.h"

#ifndef W4A16_L2_PROMOTION  // L2 fill granularity of the weight copies (CU_TENSOR_MAP_L2_PROMOTION_*)
#define W4A16_L2_PROMOTION 2  // 128 bytes (64, 128 and 256 measured within 0.2%)
#endif
#ifndef W4A16_TMA_WARPS
#define W4A16_TMA_WARPS 12
#endif
#ifndef W4A16_DECODE_WARPS  // warps of the decode-step geometry (two CTAs per SM)
#define W4A16_DECODE_WARPS 8
#endif
#ifndef W4A16_DECODE_CTAS_PER_SM  // decode geometry: CTA-local ranges per SM (1: leave room for the next kernel)
#define W4A16_DECODE_CTAS_PER_SM 1
#endif
#ifndef W4A16_TMA_STAGES
#define W4A16_TMA_STAGES 2
#endif
#ifndef W4A16_TMA_SLABS
#define W4A16_TMA_SLABS 4
#endif
#ifndef W4A16_TMA_RT
#define W4A16_TMA_RT 1
#endif


namespace w4a16 {

// First error code raised by a kernel on this device since the last read.
__device__ int g_device_error = 0;

enum DeviceErrorCode : int {
  kDevErrStageTimeout = 1,  // a TMA stage did not land within the wait limit
  kDevErrPeerTimeout = 2,   // a peer GPU's start or done flag did not arrive in time
};

// Fused all-gather (tensor parallel): every rank owns a region [header][gathered output];
// the header holds, per source rank k, a start flag and a done flag (step epochs), this
// rank's epoch, and a CTA-completion counter.  Peers write the flags through NVLink.
constexpr int kMaxRanks = 8;
constexpr int kTpStart = 0;                 // u32 [kMaxRanks]
constexpr int kTpDone = kMaxRanks;          // u32 [kMaxRanks]
constexpr int kTpEpoch = 2 * kMaxRanks;     // u32
constexpr int kTpCtaDone = 2 * kMaxRanks + 1;
// Step timeline in this rank's own header (u64 %globaltimer ns at byte 192): [0] start flags
// published, [1] every rank's start flag seen (first warp), [2] this rank's rows stored and
// fenced (done flags about to be published), [3] every rank's done flag seen.
constexpr int kTpTimeline = 48;  // u32 index: byte 192

constexpr uint64_t kStageWaitLimitNs = 2000000000ull;  // 2 s; a stage normally lands in us
constexpr uint64_t kDrainWaitLimitNs = 100000000ull;   // 0.1 s per outstanding stage

__device__ __forceinline__ void record_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

constexpr int kMaxBatchPerPass = 16;
// Workspace layout: [counters: kMaxWarps x u32][fp32 partials: kMaxWarps x 2 slots x
// batch x tile rows].  Counter w (< kMaxWarps - 2) belongs to the stream-K tile whose
// first unit warp w owns; the last two are the dynamic scheduler's next-tile and
// finished-warp counters.  Both regions have a size fixed by kMaxWarps, not by the
// problem, so calls of any shape can share one workspace.
constexpr int kMaxWarps = 4096;
constexpr size_t kCounterBytes = (size_t)kMaxWarps * 4;
constexpr int kNextTileCounter = kMaxWarps - 1;
constexpr int kDoneWarpCounter = kMaxWarps - 2;

struct TmaParams {
  const void* scale_rows;  // per-row scale [N] (group 0)
  const __half* x;         // [M][K]
  void* y;                 // [M][N]
  const float* bias;       // [N] or null
  float* partial;          // [nwarps][2][M][tile rows] (stream-K mode)
  unsigned* counters;      // [nwarps] (stream-K mode)
  long long units;         // ntiles * nwin
  int M, N, K;
  int ntiles, kslabs, nwin;
  int nwarps;              // warps that receive work
  int sched;               // kSchedStreamK, kSchedStatic or kSchedDynamic
  int slots;               // kSchedLocal: ring slots the CTA lays out (its largest unit range)
  int out_swiglu;          // rows 16b+i / 16b+8+i are a gate / up pair: y[8b+i] = silu(g) * u
  const void* pro_src;     // prologue source (XM 2: fp32 h [K]; XM 3: fp16 gate|up [2K])
  const float* pro_gamma;  // XM 2: fp32 gamma [K]
  float pro_eps;           // XM 2: epsilon
  // fused all-gather (tp_n > 1, one vector): rows go to row tp_row0 + r of every rank's
  // gathered output tp_out[k]; tp_flags[k] is rank k's header
  int tp_n, tp_rank;
  long long tp_row0;
  unsigned long long tp_wait_ns;  // limit of each wait on another rank's flags
  void* tp_out[kMaxRanks];
  unsigned* tp_flags[kMaxRanks];
};

// How the single activation vector reaches shared memory (template parameter XM):
//   kXGlobal   B fragments are loaded from global memory (no staging)
//   kXCopy     x (fp16 [K]) is copied as is
//   kXRmsNorm  x = fp16(h * rsqrt(mean(h^2) + eps) * gamma) from an fp32 vector h
//   kXSwiGlu   x = fp16(silu(g) * u) from an fp16 vector [g (K) | u (K)]
enum XMode : int { kXGlobal = 0, kXCopy = 1, kXRmsNorm = 2, kXSwiGlu = 3 };

// Work distribution over (16-row tile, 1024-column window) units:
//   kSchedStreamK  every warp takes an equal contiguous range of units; tiles shared
//                  by neighbouring warps are reduced through the workspace.  Best when
//                  there are few tiles with many windows (short, wide layers).
//   kSchedStatic   every warp takes an equal contiguous range of whole tiles (no
//                  workspace needed).
//   kSchedDynamic  warps pull whole tiles from an atomic counter in the workspace, so
//                  SMs that stream faster take more tiles.  Best for many tiles.
//   kSchedLocal    every CTA takes an equal contiguous range of whole tiles and its
//                  warps split that range's units (at most STAGES each, so every copy
//                  is issued at the start); tiles shared by warps are reduced in shared
//                  memory.  No workspace, no atomics: for the small matrices of a decode
//                  step, whose time is latency rather than bandwidth.
enum Sched : int { kSchedStreamK = 0, kSchedStatic = 1, kSchedDynamic = 2, kSchedLocal = 3 };

// 8-element chunks of the staged vector per thread (K <= kStageChunks * 8 * threads).
constexpr int kStageChunks = 8;

// Units one CTA can hold under kSchedLocal, and the shared memory of their partial sums.
template <int WARPS, int STAGES, int ROWS>
struct LocalPlan {
  static constexpr int kUnits = WARPS * STAGES;
  static constexpr int kBytes = kUnits * ROWS * 4;
};

// Offset of the staged activation after `slots` ring slots of weights, scales and
// mbarriers (WARPS * STAGES slots give SmemPlan::kXOff).  A kSchedLocal launch lays out
// only the units its CTA range holds, so that a following kernel's CTA fits on the same
// SM while this one runs.
template <typename L>
__host__ __device__ constexpr int ring_x_offset(int slots) {
  return (slots * (L::kWStride + L::kSStride + 8) + 127) / 128 * 128;
}

// Warp owning unit u of a range split [floor(w*U/T), floor((w+1)*U/T)).
__device__ __forceinline__ int warp_of_unit(long long u, long long U, int T) {
  return (int)(((u + 1) * (long long)T - 1) / U);
}

template <int PACK, int GS, typename ST, int NB, typename OT, int WARPS, int STAGES, int SLABS, int RT,
          int XM, bool TP = false>
__global__ void __launch_bounds__(WARPS * 32, WARPS == W4A16_DECODE_WARPS && WARPS <= 8 ? 2 : 1)
    k_gemv_tma(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
               const TmaParams p) {
  using L = StageLayout<SLABS, RT, GS, ST>;
  constexpr int NH = BatchCfg<NB>::kHalves;
  constexpr int kRows = L::kRows;
  static_assert(L::kScaleBoxOk, "scale box row must be a 16-byte multiple");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;  // MMA group id: rows g and g+8 of each 16-row block
  const int t = lane & 3;   // thread in group: 32-column chunk t of each 128-column group

  // XS: the CTA writes the activation vector into shared memory (fragment order,
  // see xs_offset), copying it or computing it from the prologue source; every B
  // fragment is then one shared-memory load.  The staging comes after the first
  // weight copies are in flight.
  constexpr bool XS = XM != kXGlobal;
  constexpr bool FOLD = W4A16_FOLD && NB == 1;
  constexpr bool FOLDLO = FOLD && GS && W4A16_FOLD_LO;
  constexpr bool ROWFOLD = FOLD && !GS && W4A16_ROW_NORESET;
  static_assert(ring_x_offset<L>(WARPS * STAGES) == SmemPlan<WARPS, STAGES, L>::kXOff, "ring layout");
  // after the rings: [staged x: 2K bytes if XS][128-byte scratch][FOLD corrections:
  // K/128 group floats, then (ROWFOLD) nwin window sums, 128-byte padded][kSchedLocal
  // partial sums]
  // only one-vector launches take kSchedLocal (batched ones keep the compile-time layout)
  const bool local = NB == 1 && p.sched == kSchedLocal;
  // SwiGLU epilogue (gate|up projection of a decode step): compiled into the RMSNorm kernels
  const bool swo = XM == kXRmsNorm && NB == 1 && p.out_swiglu != 0;
  // ring slots laid out: the CTA range's units under kSchedLocal, else STAGES per warp
  const int nslots = local ? p.slots : WARPS * STAGES;
  const uint32_t xs = base + (uint32_t)ring_x_offset<L>(nslots);
  const uint32_t red_off = XS ? (uint32_t)p.K * 2u : 0u;
  const uint32_t corr = xs + red_off + 128u;
  const uint32_t corr_bytes =
      FOLD ? (uint32_t)((((p.K >> 7) + (ROWFOLD ? p.nwin : 0)) * 4 + 127) & ~127) : 0u;
  const uint32_t corrw = corr + (uint32_t)(p.K >> 7) * 4u;  // ROWFOLD window sums

  const int ks = p.kslabs;
  const int nwin = p.nwin;
  // kSchedLocal: this CTA's tiles [tb0, tb0 + ntl) and their units, split over its warps
  const int tb0 = (int)((long long)blockIdx.x * p.ntiles / gridDim.x);
  const int ntl = local ? (int)((long long)(blockIdx.x + 1) * p.ntiles / gridDim.x) - tb0 : 0;
  const int gw = local ? warp : warp * gridDim.x + blockIdx.x;  // warp-major: ranges spread over all SMs
  const long long U = local ? (long long)ntl * nwin : p.units;
  const int T = local ? WARPS : p.nwarps;
  const bool active = gw < T;
  // kSchedLocal with few windows per CTA (the decode geometry, group-128, one staged vector):
  // fsplit warps share each window, warp w summing slabs [(w % fsplit) * 4 / fsplit, ...) of
  // window w / fsplit of the CTA range, so a CTA of two windows keeps 8 warps busy, not 2.
  constexpr bool kCanSplit = WARPS == W4A16_DECODE_WARPS && GS != 0 && NB == 1 && XS && SLABS == 4 && !TP;
  const int fsplit = kCanSplit && local && !swo ? (U * 4 <= WARPS ? 4 : U * 2 <= WARPS ? 2 : 1) : 1;
  const bool split = fsplit > 1;
  const int sgrp = warp / fsplit, spart = warp - sgrp * fsplit;  // window in the range, part
  const bool sgrp_ok = sgrp < U;
  const bool dyn = p.sched == kSchedDynamic;
  unsigned* next_tile = p.counters + kNextTileCounter;
  auto pull_tile = [&]() -> int {  // dynamic scheduling: the next unclaimed tile
    unsigned v = 0;
    if (lane == 0) v = atomicAdd(next_tile, 1u);
    return (int)__shfl_sync(0xffffffffu, v, 0);
  };
  long long u0, u1;
  if (p.sched == kSchedStatic) {
    u0 = (long long)gw * p.ntiles / T * nwin;
    u1 = (long long)(gw + 1) * p.ntiles / T * nwin;
  } else if (p.sched == kSchedStreamK) {
    u0 = (long long)gw * U / T;
    u1 = (long long)(gw + 1) * U / T;
  } else if (local && split) {  // the group's first warp issues its window's copy
    u0 = (long long)tb0 * nwin + sgrp;
    u1 = u0 + (spart == 0 && sgrp_ok ? 1 : 0);
  } else if (local) {  // units counted from the CTA's first tile
    u0 = (long long)tb0 * nwin + (long long)gw * U / T;
    u1 = (long long)tb0 * nwin + (long long)(gw + 1) * U / T;
  } else {
    u0 = active ? (long long)pull_tile() * nwin : U;
    u1 = u0 < U ? U : u0;  // bounded below by the tiles actually pulled
  }
  const int first_tile = (int)(u0 / nwin);
  const int first_win = (int)(u0 - (long long)first_tile * nwin);
  const int count = active ? (int)(u1 - u0) : 0;

  // [W slots: nslots x kWStride][scale slots: nslots x kSStride][mbarriers: nslots x 8].
  // A warp's ring is STAGES consecutive slots from slot0; under kSchedLocal its units
  // (count <= STAGES, no wrap) take the slots of their places in the CTA range.
  // (gw * U / T is u0 - tb0 * nwin under kSchedLocal; it does not wait for a tile claim)
  const int slot0 = local ? (split ? (sgrp_ok ? sgrp : 0) : (int)((long long)gw * U / T)) : warp * STAGES;
  const uint32_t wring = base + (uint32_t)(slot0 * L::kWStride);
  const uint32_t sring = base + (uint32_t)(nslots * L::kWStride + slot0 * L::kSStride);
  const uint32_t bar0 = base + (uint32_t)(nslots * (L::kWStride + L::kSStride) + slot0 * 8);

  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s)
      if (!local || s < count) mbar_init(bar0 + 8 * s, 1);
    mbar_fence_init();
    tma_prefetch_desc(&wmap);
    if (GS) tma_prefetch_desc(&smap);
  }
  __syncwarp();
  const uint64_t policy = l2_policy_evict_first();
  const LaneOffsets lo = lane_offsets(g, t);

  // Producer position (identical in every lane; lane 0 issues the copies).  Under
  // dynamic scheduling slot_tile remembers which tile each ring slot was filled from.
  int p_tile = first_tile, p_win = first_win;
  int issued = 0;
  bool p_done = count <= 0;
  int slot_tile[STAGES];
#pragma unroll
  for (int i = 0; i < STAGES; ++i) slot_tile[i] = first_tile;
  auto issue_one = [&]() {
    if (issued >= count || p_done) return;
    if (dyn) {
#pragma unroll
      for (int i = 0; i < STAGES; ++i)
        if ((uint32_t)issued % STAGES == (uint32_t)i) slot_tile[i] = p_tile;
    }
    const uint32_t slot = (uint32_t)issued % STAGES;
    if (lane == 0) {
      const int row0 = p_tile * kRows;
      const int s0 = p_win * SLABS;
      const uint32_t bar = bar0 + 8 * slot;
      const uint32_t dst = wring + slot * L::kWStride;
      // the full box is credited, including slabs past K that TMA fills with zeros
      mbar_arrive_expect_tx(bar, (uint32_t)(L::kWBytes + L::kSBytes));
      tma_load_3d(dst, &wmap, 0, s0, row0, bar, policy);
      if (GS) tma_load_2d(sring + slot * L::kSStride, &smap, p_win * L::kGroups, row0, bar, policy);
    }
    ++issued;
    if (++p_win == nwin) {
      p_win = 0;
      p_tile = dyn ? pull_tile() : p_tile + 1;
      if (dyn && p_tile >= p.ntiles) p_done = true;
    }
  };

#pragma unroll 1
  for (int s = 0; s < STAGES; ++s) issue_one();

  // RMSNorm: gamma is a weight, not the previous kernel's output; a thread's first chunk
  // of it is loaded before the dependency wait below.
  float4 g0[2] = {};
  if (XM == kXRmsNorm && (int)threadIdx.x < (p.K >> 3)) {
    g0[0] = __ldg(reinterpret_cast<const float4*>(p.pro_gamma) + 2 * threadIdx.x);
    g0[1] = __ldg(reinterpret_cast<const float4*>(p.pro_gamma) + 2 * threadIdx.x + 1);
  }

  // Everything above touches only the weights and this call's workspace.  Under a
  // programmatic dependent launch the previous kernel may still be running: wait for
  // it before reading the activation, the bias or anything it wrote, then let the
  // next kernel be scheduled (it will overlap this one's tail).
  grid_dependency_wait();
  grid_launch_dependents();
  // fused all-gather: per-CTA warp counter in the 128-byte scratch (bytes 64..67; the
  // RMSNorm prologue uses only its first WARPS * 4 <= 64 bytes)
  static_assert(WARPS * 4 <= 64, "scratch layout");
  unsigned& tp_warps_done = *reinterpret_cast<unsigned*>(smem_raw + (xs - smem_addr(smem_raw)) + red_off + 64);
  if (TP && p.tp_n > 1) {
    if (threadIdx.x == 0) tp_warps_done = 0u;  // a barrier follows before any warp counts
    const unsigned e = *reinterpret_cast<volatile unsigned*>(p.tp_flags[p.tp_rank] + kTpEpoch) + 1u;
    if (blockIdx.x == 0 && threadIdx.x < p.tp_n)
      st_release_sys(p.tp_flags[threadIdx.x] + kTpStart + p.tp_rank, e);
    if (blockIdx.x == 0 && threadIdx.x == 0)
      *reinterpret_cast<volatile unsigned long long*>(p.tp_flags[p.tp_rank] + kTpTimeline) = globaltimer_ns();
  }

  // kSchedLocal partial sums [unit of the CTA][16 rows] sit after the staged vector;
  // slots no segment starts at stay zero
  float* lpart = reinterpret_cast<float*>(smem_raw + (corr - smem_addr(smem_raw)) + corr_bytes);
  if (local) {
    for (int i = threadIdx.x; i < LocalPlan<WARPS, STAGES, kRows>::kUnits * kRows; i += blockDim.x)
      lpart[i] = 0.f;
    if (!XS) __syncthreads();
  }

  // FOLD: corr[g] = -72 * (sum of the fp16 activation over the columns whose codes
  // decode_word_fold leaves biased: 8i+2, 8i+3, 8i+6, 8i+7 of group g for the interleaved
  // packing, the even columns 8i, 8i+2, 8i+4, 8i+6 for the simple one) (FOLDLO: minus
  // 1032 * the sum over columns 8i, 8i+1, 8i+4, 8i+5 as well), summed by the 16 threads
  // holding the group's 16 chunks (a thread's chunks are warp-uniformly in or out of
  // range: K is a multiple of 256).
  const int nch = p.K >> 3;  // 8-element chunks; thread i takes chunks i, i + blockDim, ...
  float* corr_f = reinterpret_cast<float*>(smem_raw + (corr - smem_addr(smem_raw)));
  auto fold_correction = [&](int c, const uint4& v) {
    float part;
    if (PACK == W4A16_PACK_SIMPLE) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
      const float2 c2 = __half22float2(*reinterpret_cast<const __half2*>(&v.z));
      const float2 d2 = __half22float2(*reinterpret_cast<const __half2*>(&v.w));
      part = (a.x + b.x) + (c2.x + d2.x);
    } else {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.w));
      part = (a.x + a.y) + (b.x + b.y);
    }
    float part_lo = 0.f;
    if (FOLDLO) {
      const float2 c2 = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
      const float2 d2 = __half22float2(*reinterpret_cast<const __half2*>(&v.z));
      part_lo = (c2.x + c2.y) + (d2.x + d2.y);
    }
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
      part += __shfl_xor_sync(0xffffffffu, part, o);
      if (FOLDLO) part_lo += __shfl_xor_sync(0xffffffffu, part_lo, o);
    }
    if ((lane & 15) == 0 && c < nch) corr_f[c >> 4] = FOLDLO ? -72.f * part - 1032.f * part_lo : -72.f * part;
  };
  // ROWFOLD: corr_f[K/128 + w] = sum of the corrections of window w's groups
  auto window_corrections = [&]() {
    const int ng = p.K >> 7;
    for (int w = threadIdx.x; w < p.nwin; w += blockDim.x) {
      float sum = 0.f;
      for (int gi = w * 2 * SLABS; gi < ng && gi < (w + 1) * 2 * SLABS; ++gi) sum += corr_f[gi];
      corr_f[ng + w] = sum;
    }
    __syncthreads();
  };
  if (FOLD && !XS) {  // the vector stays in global memory: read it once for the sums
    for (int c0 = 0; c0 < nch; c0 += blockDim.x) {
      const int c = c0 + threadIdx.x;
      const uint4 v = c < nch ? ldcg128(p.x + c * 8) : make_uint4(0u, 0u, 0u, 0u);
      fold_correction(c, v);
    }
    __syncthreads();
    if (ROWFOLD) window_corrections();
  }

  if (XS) {
    // x, h, gate|up and the bias may have been written by the previous kernel:
    // read them through L2 (ldcg), not the non-coherent path.
    uint8_t* xsp = smem_raw + (xs - smem_addr(smem_raw));
    // Every loop below is unrolled over kStageChunks chunks per thread with a guard, so a
    // thread's loads are all in flight together (the host stages only K <= kStageChunks *
    // threads * 8).
    if (XM == kXCopy) {
#pragma unroll
      for (int j = 0; j < kStageChunks; ++j) {
        const int c = threadIdx.x + j * WARPS * 32;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (c < nch) {
          v = ldcg128(p.x + c * 8);
          *reinterpret_cast<uint4*>(xsp + xs_offset(c * 8)) = PACK == W4A16_PACK_SIMPLE ? simple_order(v) : v;
        }
        if (FOLD) fold_correction(c, v);
      }
    } else if (XM == kXRmsNorm) {
      const float4* h4 = static_cast<const float4*>(p.pro_src);
      const float4* g4 = reinterpret_cast<const float4*>(p.pro_gamma);
      // A thread's first chunk of h stays in registers for the second pass (and its first
      // chunk of gamma is already there), so a vector of at most one chunk per thread
      // costs one round trip to L2, not two.
      float4 h0[2] = {};
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < kStageChunks; ++j) {
        const int c = threadIdx.x + j * WARPS * 32;
        if (c < nch) {
          const float4 a = __ldcg(h4 + 2 * c), b = __ldcg(h4 + 2 * c + 1);
          if (j == 0) {
            h0[0] = a;
            h0[1] = b;
          }
          ss = fmaf(a.x, a.x, ss);
          ss = fmaf(a.y, a.y, ss);
          ss = fmaf(a.z, a.z, ss);
          ss = fmaf(a.w, a.w, ss);
          ss = fmaf(b.x, b.x, ss);
          ss = fmaf(b.y, b.y, ss);
          ss = fmaf(b.z, b.z, ss);
          ss = fmaf(b.w, b.w, ss);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      float* red = reinterpret_cast<float*>(xsp + red_off);  // WARPS partial sums
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) tot += red[w];
      const float r = rsqrtf(tot / (float)p.K + p.pro_eps);
#pragma unroll
      for (int j = 0; j < kStageChunks; ++j) {
        const int c = threadIdx.x + j * WARPS * 32;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (c < nch) {
          const float4 a = j == 0 ? h0[0] : __ldcg(h4 + 2 * c), b = j == 0 ? h0[1] : __ldcg(h4 + 2 * c + 1);
          const float4 ga = j == 0 ? g0[0] : __ldg(g4 + 2 * c), gb = j == 0 ? g0[1] : __ldg(g4 + 2 * c + 1);
          v.x = pack_half2(a.x * r * ga.x, a.y * r * ga.y);
          v.y = pack_half2(a.z * r * ga.z, a.w * r * ga.w);
          v.z = pack_half2(b.x * r * gb.x, b.y * r * gb.y);
          v.w = pack_half2(b.z * r * gb.z, b.w * r * gb.w);
          *reinterpret_cast<uint4*>(xsp + xs_offset(c * 8)) = PACK == W4A16_PACK_SIMPLE ? simple_order(v) : v;
        }
        if (FOLD) fold_correction(c, v);
      }
    } else if (XM == kXSwiGlu) {
      const __half* gu = static_cast<const __half*>(p.pro_src);
#pragma unroll
      for (int j = 0; j < kStageChunks; ++j) {
        const int c = threadIdx.x + j * WARPS * 32;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (c < nch) {
          const uint4 gv = ldcg128(gu + c * 8);
          const uint4 uv = ldcg128(gu + p.K + c * 8);
          const uint32_t gw4[4] = {gv.x, gv.y, gv.z, gv.w};
          const uint32_t uw4[4] = {uv.x, uv.y, uv.z, uv.w};
          uint32_t pk[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 g2 = __half22float2(*reinterpret_cast<const __half2*>(&gw4[i]));
            const float2 u2 = __half22float2(*reinterpret_cast<const __half2*>(&uw4[i]));
            pk[i] = pack_half2(silu_mul(g2.x, u2.x), silu_mul(g2.y, u2.y));
          }
          v = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(xsp + xs_offset(c * 8)) = PACK == W4A16_PACK_SIMPLE ? simple_order(v) : v;
        }
        if (FOLD) fold_correction(c, v);
      }
    }
    __syncthreads();
    if (ROWFOLD) window_corrections();
  }

  // Fused all-gather.  CTA 0 announces step tp_e to every rank (the previous kernel has
  // completed, so this rank is done with the previous gathered output).  Each warp, before
  // its first store into other ranks' buffers, waits until every rank has announced the
  // step; the last warp of the last CTA publishes this rank's done flag to every rank,
  // waits for all of theirs and advances this rank's epoch, so the kernel completes only
  // when the whole gathered output is in place.  Every wait gives up after 2 s, records the
  // error, and the warp then writes this rank's own buffer only.
  const bool tp = TP && p.tp_n > 1;  // the fused all-gather is compiled only into TP kernels
  unsigned* tp_my = tp ? p.tp_flags[p.tp_rank] : nullptr;
  const unsigned tp_e = tp ? *reinterpret_cast<volatile unsigned*>(tp_my + kTpEpoch) + 1u : 0u;
  bool tp_started = false, tp_peers_ok = false;
  auto tp_ensure_started = [&]() {  // warp-uniform
    if (!tp || tp_started) return;
    int ok = 1;
    if (lane == 0) {
      const uint64_t t0 = globaltimer_ns();
      for (int k = 0; k < p.tp_n && ok; ++k)
        while ((int)(ld_acquire_sys(tp_my + kTpStart + k) - tp_e) < 0) {
          if (globaltimer_ns() - t0 > p.tp_wait_ns) {
            record_device_error(kDevErrPeerTimeout);
            ok = 0;
            break;
          }
        }
    }
    if (lane == 0 && blockIdx.x == 0 && warp == 0)
      *reinterpret_cast<volatile unsigned long long*>(tp_my + kTpTimeline + 2) = globaltimer_ns();
    tp_peers_ok = __shfl_sync(0xffffffffu, ok, 0) != 0;
    tp_started = true;
  };
  // One output element: the plain output, or row tp_row0 + r of every rank's buffer.
  auto store_out = [&](size_t idx, int r, float v) {
    if (!tp) {
      static_cast<OT*>(p.y)[idx] = from_f32<OT>(v);
      return;
    }
    const OT ov = from_f32<OT>(v);
    if (tp_peers_ok) {
      for (int k = 0; k < p.tp_n; ++k) static_cast<OT*>(p.tp_out[k])[p.tp_row0 + r] = ov;
    } else {
      static_cast<OT*>(p.tp_out[p.tp_rank])[p.tp_row0 + r] = ov;
    }
  };
  auto tp_warp_done = [&]() {
    if (!tp) return;
    __syncwarp();
    if (lane == 0) {
      // Release chain: each warp's stores are ordered before its count (GPU-scope fence);
      // the CTA's last warp, having observed every count, makes them visible at system
      // scope before the grid-wide count, and the last CTA once more before the flags.
      // (One system-scope fence per CTA instead of per warp: 68.2 -> 65.4 us per 2-GPU
      // step.)
      __threadfence();
      if (atomicAdd(&tp_warps_done, 1u) == (unsigned)(WARPS - 1) &&
          (__threadfence_system(), atomicAdd(tp_my + kTpCtaDone, 1u) == gridDim.x - 1)) {
        tp_my[kTpCtaDone] = 0u;
        __threadfence_system();
        *reinterpret_cast<volatile unsigned long long*>(tp_my + kTpTimeline + 4) = globaltimer_ns();
        for (int k = 0; k < p.tp_n; ++k) st_release_sys(p.tp_flags[k] + kTpDone + p.tp_rank, tp_e);
        const uint64_t t0 = globaltimer_ns();
        for (int k = 0; k < p.tp_n; ++k)
          while ((int)(ld_acquire_sys(tp_my + kTpDone + k) - tp_e) < 0) {
            if (globaltimer_ns() - t0 > p.tp_wait_ns) {
              record_device_error(kDevErrPeerTimeout);
              break;
            }
          }
        *reinterpret_cast<volatile unsigned long long*>(tp_my + kTpTimeline + 6) = globaltimer_ns();
        tp_my[kTpEpoch] = tp_e;
      }
    }
  };

  if (kCanSplit && split) {
    // The window's mbarrier was initialised by its issuing warp before the staging barrier.
    float tot[RT][NH][4], acc[RT][2][NH][4];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i) tot[rt][h][i] = acc[rt][0][h][i] = acc[rt][1][h][i] = 0.f;
    if (sgrp_ok) {
      if (!mbar_wait_bounded(bar0, 0u, kStageWaitLimitNs)) {
        record_device_error(kDevErrStageTimeout);
        if (spart == 0) mbar_wait_bounded(bar0, 0u, kDrainWaitLimitNs);  // its copy may still land
      } else {
        const int win = (int)(sgrp % nwin);
        const int s0 = win * SLABS;
        const int sa = spart * (SLABS / fsplit), sb = min(sa + SLABS / fsplit, ks - s0);
        if (sb > sa)
          consume_window<false, XS, PACK, GS, ST, NB, RT, SLABS, FOLD, FOLDLO>(
              wring, sring, xs, corr, sb, s0 * kSlabCols, p.x, p.K, p.M, g, t, lo, acc, tot, sa);
      }
      float* lp = lpart + ((long long)sgrp * fsplit + spart) * kRows;  // [window][part][rows]
      if (t == 0) {
#pragma unroll
        for (int rt = 0; rt < RT; ++rt) {
          lp[rt * 16 + g] = tot[rt][0][0];
          lp[rt * 16 + g + 8] = tot[rt][0][2];
        }
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < ntl * kRows; i += blockDim.x) {  // windows and parts in order
      const int tl = i / kRows, rl = i - tl * kRows;
      const int r = (tb0 + tl) * kRows + rl;
      if (r >= p.N) continue;
      float v = 0.f;
      for (int w = 0; w < nwin * fsplit; ++w) v += lpart[((long long)tl * nwin * fsplit + w) * kRows + rl];
      if (p.bias) v += __ldcg(p.bias + r);
      store_out(r, r, v);
    }
    return;
  }

  if (!active && !local) {
    tp_warp_done();
    return;
  }

  float tot[RT][NH][4];
  float acc[RT][2][NH][4];
  uint32_t srow_bits[RT][2];  // per-row scales (raw bits), converted in the epilogue
  float csum = 0.f;           // ROWFOLD: bias correction of the segment's windows
  int tile = first_tile, win = first_win, tile_w0 = first_win;

#pragma unroll 1
  for (int consumed = 0; consumed < count; ++consumed) {
    if (dyn) {
      if (consumed >= issued) break;  // the producer has run out of tiles
#pragma unroll
      for (int i = 0; i < STAGES; ++i)
        if ((uint32_t)consumed % STAGES == (uint32_t)i) tile = slot_tile[i];
    }
    if (win == 0 || consumed == 0) {  // a tile starts in this warp's range
      tile_w0 = win;
      csum = 0.f;
#pragma unroll
      for (int rt = 0; rt < RT; ++rt) {
#pragma unroll
        for (int h = 0; h < NH; ++h)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            tot[rt][h][i] = 0.f;
            acc[rt][0][h][i] = 0.f;
            acc[rt][1][h][i] = 0.f;
          }
        const int r0 = tile * kRows + rt * 16 + g;
        if (!GS) {  // per-row scales are used in the epilogue: issue the loads now
          const ST* sr = static_cast<const ST*>(p.scale_rows);
          srow_bits[rt][0] = r0 < p.N ? ld_scale_bits_now<ST>(sr + r0) : 0u;
          srow_bits[rt][1] = r0 + 8 < p.N ? ld_scale_bits_now<ST>(sr + r0 + 8) : 0u;
        }
      }
    }

    const uint32_t slot = (uint32_t)consumed % STAGES;
    const uint32_t parity = ((uint32_t)consumed / STAGES) & 1u;
    if (!mbar_wait_bounded(bar0 + 8 * slot, parity, kStageWaitLimitNs)) {
      record_device_error(kDevErrStageTimeout);
      for (int s = consumed + 1; s < issued; ++s)
        mbar_wait_bounded(bar0 + 8 * (s % STAGES), (s / STAGES) & 1u, kDrainWaitLimitNs);
      if (local) break;  // the CTA still meets at the reduction barrier
      tp_warp_done();
      return;
    }
    const uint32_t wbase = wring + slot * L::kWStride;
    const uint32_t sbase = sring + slot * L::kSStride;
    const int s0 = win * SLABS;
    const int nslab = min(SLABS, ks - s0);
    if (ROWFOLD) csum += lds_f32(corrw + (uint32_t)win * 4u);
    if (nslab == SLABS)
      consume_window<true, XS, PACK, GS, ST, NB, RT, SLABS, FOLD, FOLDLO>(
          wbase, sbase, xs, corr, nslab, s0 * kSlabCols, p.x, p.K, p.M, g, t, lo, acc, tot);
    else
      consume_window<false, XS, PACK, GS, ST, NB, RT, SLABS, FOLD, FOLDLO>(
          wbase, sbase, xs, corr, nslab, s0 * kSlabCols, p.x, p.K, p.M, g, t, lo, acc, tot);
    __syncwarp();  // every lane has read the slot before it is refilled
    issue_one();

    const int cur_tile = tile;
    const bool tile_done = win == nwin - 1;
    if (++win == nwin) {
      win = 0;
      ++tile;
    }
    if (!tile_done && (dyn || consumed + 1 < count)) continue;  // the tile goes on here

    // ---- tile epilogue
    float srow[RT][2];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt) {
      srow[rt][0] = GS ? 1.f : scale_from_bits<ST>(srow_bits[rt][0]);
      srow[rt][1] = GS ? 1.f : scale_from_bits<ST>(srow_bits[rt][1]);
    }
    if (ROWFOLD) {  // one accumulation per segment, minus the windows' bias
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          tot[rt][h][0] = (acc[rt][0][h][0] + acc[rt][1][h][0] + csum) * srow[rt][0];
          tot[rt][h][2] = (acc[rt][0][h][2] + acc[rt][1][h][2] + csum) * srow[rt][1];
        }
    } else if (!GS && FOLD) {  // the groups were summed into tot: apply the row scale
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          tot[rt][h][0] *= srow[rt][0];
          tot[rt][h][1] *= srow[rt][0];
          tot[rt][h][2] *= srow[rt][1];
          tot[rt][h][3] *= srow[rt][1];
        }
    } else if (!GS) {
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          tot[rt][h][0] = (acc[rt][0][h][0] + acc[rt][1][h][0]) * srow[rt][0];
          tot[rt][h][1] = (acc[rt][0][h][1] + acc[rt][1][h][1]) * srow[rt][0];
          tot[rt][h][2] = (acc[rt][0][h][2] + acc[rt][1][h][2]) * srow[rt][1];
          tot[rt][h][3] = (acc[rt][0][h][3] + acc[rt][1][h][3]) * srow[rt][1];
        }
    }
    // Fragment (rt, h, i): row cur_tile*kRows + rt*16 + g (+8 for i >= 2), batch
    // column n = h*8 + 2t + (i & 1).
    if (swo && tile_w0 == 0 && tile_done) {  // rows g and g + 8 of each block: a gate / up pair
#pragma unroll
      for (int rt = 0; rt < RT; ++rt) {
        const int r0 = cur_tile * kRows + rt * 16;
        if (t == 0 && r0 < p.N) store_out(r0 / 2 + g, r0 / 2 + g, silu_mul(tot[rt][0][0], tot[rt][0][2]));
      }
      continue;
    }
    if (tile_w0 == 0 && tile_done) {  // the whole tile was summed here
      tp_ensure_started();
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int h = 0; h < NH; ++h)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = cur_tile * kRows + rt * 16 + g + (i < 2 ? 0 : 8);
            const int n = h * 8 + 2 * t + (i & 1);
            const bool ok = NB == 1 ? (t == 0 && (i & 1) == 0) : (n < p.M);
            if (ok && r < p.N) {
              float v = tot[rt][h][i];
              if (p.bias) v += __ldcg(p.bias + r);  // may be the previous kernel's output
              store_out((size_t)n * p.N + r, r, v);
            }
          }
      continue;
    }
    if (local) {  // segment of a tile shared within the CTA: its partial goes to smem
      float* lp = lpart + ((cur_tile - tb0) * nwin + tile_w0) * kRows;
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int h = 0; h < NH; ++h)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const bool ok = NB == 1 && t == 0 && (i & 1) == 0;
            if (ok) lp[rt * 16 + g + (i < 2 ? 0 : 8)] = tot[rt][h][i];
          }
      continue;
    }
    // Part of a tile shared with neighbouring warps: publish the partial sums; the
    // last contributor adds all of them in warp order and writes the tile.
    const int slot_out = cur_tile == first_tile ? 0 : 1;
    float* mine = p.partial + ((size_t)gw * 2 + slot_out) * p.M * kRows;
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rl = rt * 16 + g + (i < 2 ? 0 : 8);
          const int n = h * 8 + 2 * t + (i & 1);
          const bool ok = NB == 1 ? (t == 0 && (i & 1) == 0) : (n < p.M);
          if (ok) mine[(size_t)n * kRows + rl] = tot[rt][h][i];
        }
    const long long tu0 = (long long)cur_tile * nwin;
    const int w_first = warp_of_unit(tu0, U, T);
    const int w_last = warp_of_unit(tu0 + nwin - 1, U, T);
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(p.counters + w_first, 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != (unsigned)(w_last - w_first)) continue;
    __threadfence();
    tp_ensure_started();
    // Every contributor after the first starts inside this tile, so the tile is its
    // first (slot 0); the first contributor used slot 1 unless it also started here.
    const int slot_first = ((long long)w_first * U / T) / nwin == cur_tile ? 0 : 1;
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rl = rt * 16 + g + (i < 2 ? 0 : 8);
          const int r = cur_tile * kRows + rl;
          const int n = h * 8 + 2 * t + (i & 1);
          const bool ok = NB == 1 ? (t == 0 && (i & 1) == 0) : (n < p.M);
          if (ok && r < p.N) {
            const size_t off = (size_t)n * kRows + rl;
            const size_t wstride = (size_t)2 * p.M * kRows;
            float v = __ldcg(p.partial + ((size_t)w_first * 2 + slot_first) * p.M * kRows + off);
            for (int w = w_first + 1; w <= w_last; ++w) v += __ldcg(p.partial + (size_t)w * wstride + off);
            if (p.bias) v += __ldcg(p.bias + r);  // may be the previous kernel's output
            store_out((size_t)n * p.N + r, r, v);
          }
        }
    __syncwarp();
    if (lane == 0) p.counters[w_first] = 0u;  // leave the workspace zeroed
  }
  if (local) {
    // Tiles split between warps of this CTA: add their segments in window order.
    if constexpr (NB == 1) {
      __syncthreads();
      tp_ensure_started();
      if (swo) {  // gate / up pairs (rows 16b + i, 16b + 8 + i) -> output 8b + i
        for (int i = threadIdx.x; i < ntl * (kRows / 2); i += blockDim.x) {
          const int tl = i / (kRows / 2), pr = i - tl * (kRows / 2);
          const int rl = (pr >> 3) * 16 + (pr & 7);  // gate row in the tile; its up row is rl + 8
          const long long tu0 = (long long)tl * nwin;
          if (warp_of_unit(tu0, U, T) == warp_of_unit(tu0 + nwin - 1, U, T)) continue;  // written
          const int r = (tb0 + tl) * kRows + rl;
          if (r >= p.N) continue;
          float vg = 0.f, vu = 0.f;
          for (int w = 0; w < nwin; ++w) {
            vg += lpart[(tl * nwin + w) * kRows + rl];
            vu += lpart[(tl * nwin + w) * kRows + rl + 8];
          }
          const int o = (tb0 + tl) * (kRows / 2) + pr;
          store_out(o, o, silu_mul(vg, vu));
        }
        tp_warp_done();
        return;
      }
      for (int i = threadIdx.x; i < ntl * kRows; i += blockDim.x) {
        const int tl = i / kRows, rl = i - tl * kRows;
        const long long tu0 = (long long)tl * nwin;
        if (warp_of_unit(tu0, U, T) == warp_of_unit(tu0 + nwin - 1, U, T)) continue;  // written
        const int r = (tb0 + tl) * kRows + rl;
        if (r >= p.N) continue;
        float v = 0.f;
        for (int w = 0; w < nwin; ++w) v += lpart[(tl * nwin + w) * kRows + rl];
        if (p.bias) v += __ldcg(p.bias + r);
        store_out(r, r, v);
      }
    }
    tp_warp_done();
    return;
  }
  if (dyn && lane == 0) {
    // Every warp has made its last pull before it counts itself done, so the last
    // one can rewind the tile counter for the next call.
    if (atomicAdd(p.counters + kDoneWarpCounter, 1u) == (unsigned)(T - 1)) {
      *next_tile = 0u;
      p.counters[kDoneWarpCounter] = 0u;
    }
  }
  tp_warp_done();
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
constexpr int kRT = W4A16_TMA_RT;
constexpr int kTileRows = kMmaRows * kRT;

// CTA geometry.  The default: 12 warps, 16-row tiles.  WIDE (9..16 activation rows on a
// matrix of many tiles): every activation fragment a lane loads (from L1: the batch does not
// fit shared memory beside the rings) feeds RT = 2 row blocks, halving the activation
// traffic per weight byte that made the L1 pipe the limiter (lm_head-sized matrices at
// batch 16: 161 -> 116 us); 6 warps with 32-row stages keep the same bytes in flight.  Fewer
// warps and tiles lose on small matrices, which keep the default.
#ifndef W4A16_BATCH_WARPS
#define W4A16_BATCH_WARPS 6
#endif
#ifndef W4A16_BATCH_RT
#define W4A16_BATCH_RT 2
#endif
// LONG (one activation vector whose length does not fit shared memory beside 12 warps'
// rings): 9 warps, so that the vector is still staged in shared memory (Llama-3-8B's down
// projection, 14336 columns; its fragments otherwise come from L1 one by one).
#ifndef W4A16_LONGK_WARPS
#define W4A16_LONGK_WARPS 9
#endif
// DECODE (a staged one-vector launch whose whole matrix fits its CTAs' rings at once, as in
// a decode step): W4A16_DECODE_WARPS warps capped at 128 registers (two CTAs per SM) with
// only the ring slots their units need, so that the next chained kernel's CTA is resident
// beside this one and streams its weights while this one runs.
static_assert(W4A16_DECODE_WARPS <= 16 && W4A16_DECODE_WARPS != kWarps &&
                  W4A16_DECODE_WARPS != W4A16_BATCH_WARPS && W4A16_DECODE_WARPS != W4A16_LONGK_WARPS,
              "the two-CTA register bound goes by warp count");
enum GeometryKind : int { kGeoDefault = 0, kGeoWide = 1, kGeoLong = 2, kGeoDecode = 3 };
template <int GEO>
struct Geometry {
  static constexpr int kW = GEO == kGeoWide     ? W4A16_BATCH_WARPS
                            : GEO == kGeoLong   ? W4A16_LONGK_WARPS
                            : GEO == kGeoDecode ? W4A16_DECODE_WARPS
                                                : kWarps;
  static constexpr int kS = kStages;
  static constexpr int kR = GEO == kGeoWide ? W4A16_BATCH_RT : kRT;
  static constexpr int kTile = kMmaRows * kR;
};
constexpr int kMaxTileRows = kMmaRows * (W4A16_BATCH_RT > W4A16_TMA_RT ? W4A16_BATCH_RT : W4A16_TMA_RT);

template <int GS, typename ST, int GEO = kGeoDefault>
constexpr int tma_smem_bytes() {
  using G = Geometry<GEO>;
  using L = StageLayout<kSlabs, G::kR, GS, ST>;
  return SmemPlan<G::kW, G::kS, L>::kBytes;
}

// Shared memory after the weight/scale rings (the kernel's layout): the staged vector,
// a 128-byte scratch, the FOLD corrections; kSchedLocal adds its partial sums.
template <int PACK, int NB, int XM>
int tail_smem_bytes(int K) {
  constexpr bool fold = W4A16_FOLD && NB == 1;
  // group corrections, plus one sum per 1024-column window (read by the per-row kernels)
  const int corr = fold ? ((K / 128 + (K + 1023) / 1024) * 4 + 127) / 128 * 128 : 0;
  return (XM != kXGlobal ? K * 2 : 0) + (NB == 1 ? 128 : 0) + corr;
}

template <int PACK, int GS, typename ST, int NB, typename OT, int XM, bool TP = false, int GEO = kGeoDefault>
int launch_tma(const GemvProblem& p, const __half* x, int M, void* y, const DeviceInfo& di, int dev) {
  using G = Geometry<GEO>;
  constexpr int kWarps = G::kW;      // this launch's geometry (shadows the batch-1 defaults)
  constexpr int kStages = G::kS;
  constexpr int kRT = G::kR;
  constexpr int kTileRows = G::kTile;
  using L = StageLayout<kSlabs, kRT, GS, ST>;
  auto kernel = k_gemv_tma<PACK, GS, ST, NB, OT, kWarps, kStages, kSlabs, kRT, XM, TP>;
  // full rings; a kSchedLocal launch lays out only its units (checked below)
  const int smem_base = tma_smem_bytes<GS, ST, GEO>() + tail_smem_bytes<PACK, NB, XM>(p.K);
  int smem = smem_base;
  static std::atomic<uint64_t> configured{0};
  const uint64_t bit = 1ull << dev;
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, di.smem_optin);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(%d bytes): %s", di.smem_optin, cudaGetErrorString(e));
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
  CUresult r;
  {  // 3-D view {128 bytes, K/256 slabs, N rows}: one box [rows][SLABS][128 B] per window
    const cuuint64_t dims[3] = {128, (cuuint64_t)(p.K / kSlabCols), (cuuint64_t)p.N};
    const cuuint64_t strides[2] = {128, (cuuint64_t)(p.K / 2)};
    const cuuint32_t box[3] = {128, (cuuint32_t)kSlabs, (cuuint32_t)kTileRows};
    const cuuint32_t estr[3] = {1, 1, 1};
    r = enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(p.packed), dims, strides,
            box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            (CUtensorMapL2promotion)W4A16_L2_PROMOTION, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled(weights) failed: %d", (int)r);
      return W4A16_ERR_CUDA;
    }
  }
  if constexpr (GS != 0) {
    const int ng = p.K / GS;
    const cuuint64_t dims[2] = {(cuuint64_t)ng, (cuuint64_t)p.N};
    const cuuint64_t strides[1] = {(cuuint64_t)ng * sizeof(ST)};
    const cuuint32_t box[2] = {(cuuint32_t)L::kGroups, (cuuint32_t)kTileRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt =
        sizeof(ST) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    r = enc(&smap, dt, 2, const_cast<void*>(p.scale), dims, strides, box, estr,
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
  prm.kslabs = p.K / kSlabCols;
  prm.nwin = (prm.kslabs + kSlabs - 1) / kSlabs;
  prm.units = (long long)prm.ntiles * prm.nwin;
  const long long slots = (long long)di.sms * kWarps;
  const long long tk = prm.units < slots ? prm.units : slots;           // stream-K warps
  const long long tt = prm.ntiles < slots ? prm.ntiles : slots;         // whole-tile warps
  const size_t need = kCounterBytes + (size_t)tk * 2 * M * kTileRows * 4;
  const bool have_ws = p.split_k != 1 && tk <= kMaxWarps - 2 && p.workspace &&
                       p.workspace_bytes >= need && aligned(p.workspace, 256);
  // kSchedLocal when every CTA's share of whole tiles fits its warps' rings at once
  using LP = LocalPlan<kWarps, kStages, kTileRows>;
  const int local_ctas = di.sms * (GEO == kGeoDecode ? W4A16_DECODE_CTAS_PER_SM : 1);
  const int g_local = prm.ntiles < local_ctas ? prm.ntiles : local_ctas;
  const long long tiles_per_cta = (prm.ntiles + g_local - 1) / (g_local > 0 ? g_local : 1);
  const bool local_fit = g_local > 0 && tiles_per_cta * prm.nwin <= LP::kUnits;
  const int local_smem = local_fit ? ring_x_offset<L>((int)(tiles_per_cta * prm.nwin)) + 1024 +
                                         tail_smem_bytes<PACK, NB, XM>(p.K) + LP::kBytes
                                   : 0;
  const bool local_ok = NB == 1 && M == 1 && p.split_k != 1 && local_fit && local_smem <= di.smem_optin;
  if (local_ok)
    prm.sched = kSchedLocal;
  else if (!have_ws)
    prm.sched = kSchedStatic;
  else if (prm.ntiles * 4 >= slots || prm.nwin <= 2 || p.out_swiglu)  // whole tiles per warp
    prm.sched = kSchedDynamic;
  else
    prm.sched = kSchedStreamK;
  prm.nwarps = (int)(prm.sched == kSchedStreamK ? tk : prm.sched == kSchedLocal ? g_local * kWarps : tt);
  prm.slots = kWarps * kStages;
  if (prm.sched == kSchedLocal) {
    // every CTA range holds at most tiles_per_cta * nwin units (<= kWarps * kStages)
    prm.slots = (int)(tiles_per_cta * prm.nwin);
    smem = local_smem;
  }
  if (smem > di.smem_optin) {
    set_error("shared memory %d exceeds the device limit %d", smem, di.smem_optin);
    return W4A16_ERR_SHAPE;
  }
  prm.out_swiglu = p.out_swiglu ? 1 : 0;
  prm.pro_src = p.pro_src;
  prm.pro_gamma = p.pro_gamma;
  prm.pro_eps = p.pro_eps;
  prm.tp_n = p.tp_n;
  prm.tp_rank = p.tp_rank;
  prm.tp_row0 = p.tp_row0;
  prm.tp_wait_ns = p.tp_wait_ns;
  for (int k = 0; k < kMaxRanks; ++k) {
    prm.tp_out[k] = p.tp_out[k];
    prm.tp_flags[k] = p.tp_flags[k];
  }
  prm.partial = nullptr;
  prm.counters = nullptr;
  if (have_ws && prm.sched != kSchedLocal) {
    uint8_t* ws = static_cast<uint8_t*>(p.workspace);
    prm.counters = reinterpret_cast<unsigned*>(ws);
    prm.partial = reinterpret_cast<float*>(ws + kCounterBytes);
  }
  int grid = prm.sched == kSchedLocal ? g_local : prm.nwarps < di.sms ? prm.nwarps : di.sms;
  if (grid < 1) grid = 1;
  const cudaError_t le = launch_maybe_pdl(kernel, dim3(grid), dim3(kWarps * 32), (size_t)smem, p.stream,
                                          p.pdl, wmap, smap, prm);
  (void)cudaGetLastError();  // the status is `le`; do not leave it for a later check
  if (le != cudaSuccess) {
    set_error("k_gemv_tma launch failed: %s", cudaGetErrorString(le));
    return W4A16_ERR_CUDA;
  }
  return W4A16_OK;
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


// Whether a one-vector launch of geometry GEO takes kSchedLocal (launch_tma's test on tiles).
template <int GEO>
bool local_fits(const GemvProblem& p, const DeviceInfo& di) {
  using G = Geometry<GEO>;
  const long long ntiles = (p.N + G::kTile - 1) / G::kTile;
  const long long nwin = (p.K / kSlabCols + kSlabs - 1) / kSlabs;
  const long long ctas = (long long)di.sms * (GEO == kGeoDecode ? W4A16_DECODE_CTAS_PER_SM : 1);
  const long long g_local = ntiles < ctas ? ntiles : ctas;
  return p.split_k != 1 && g_local > 0 && (ntiles + g_local - 1) / g_local * nwin <= (long long)G::kW * G::kS;
}

template <int PACK, int GS, typename ST, typename OT>
int run_pass(const GemvProblem& p, const __half* x, int M, void* y, bool use_tma,
             const DeviceInfo& di, int dev) {
  // The simple packing (the reference's ladder kernels) only ever carries per-row
  // fp32 scales and fp32 outputs there; other combinations take the generic kernel.
  constexpr bool kTmaVariant =
      (PACK == W4A16_PACK_INTERLEAVED ||
       (GS == 0 && std::is_same<ST, float>::value && std::is_same<OT, float>::value)) &&
      StageLayout<kSlabs, kRT, GS, ST>::kScaleBoxOk;
  if (p.tp_n > 1 && (!kTmaVariant || !use_tma || M != 1 || PACK != W4A16_PACK_INTERLEAVED)) {
    set_error("the fused all-gather needs one activation vector on the TMA path: cols %% 256 == 0, "
              "16-byte aligned weights, interleaved packing");
    return W4A16_ERR_SHAPE;
  }
  if (p.staged && (!kTmaVariant || !use_tma)) {
    set_error("the staged (fused) GEMV needs the TMA path: cols %% 256 == 0, 16-byte aligned "
              "weights, interleaved packing");
    return W4A16_ERR_SHAPE;
  }
  if constexpr (!kTmaVariant) {
    (void)use_tma;
    (void)di;
    (void)dev;
    return launch_generic<PACK, GS, ST, OT>(p, x, M, y);
  } else {
  if (!use_tma) return launch_generic<PACK, GS, ST, OT>(p, x, M, y);
  const bool xs_fits = tma_smem_bytes<GS, ST>() + tail_smem_bytes<PACK, 1, kXCopy>(p.K) <= di.smem_optin &&
                       p.K <= kStageChunks * 8 * kWarps * 32;
  if (p.staged) {
    if (M != 1 || !xs_fits) {
      int kmax = kStageChunks * 8 * kWarps * 32;
      while (kmax > 0 && tma_smem_bytes<GS, ST>() + tail_smem_bytes<PACK, 1, kXCopy>(kmax) > di.smem_optin)
        kmax -= 256;
      set_error("the staged (fused) GEMV needs one activation vector and cols <= %d", kmax);
      return W4A16_ERR_SHAPE;
    }
    if constexpr (PACK == W4A16_PACK_INTERLEAVED) {
      const bool dec = local_fits<kGeoDecode>(p, di) &&
                       p.K <= kStageChunks * 8 * Geometry<kGeoDecode>::kW * 32;
      if (p.prologue == W4A16_PROLOGUE_RMSNORM)
        return dec ? launch_tma<PACK, GS, ST, 1, OT, kXRmsNorm, false, kGeoDecode>(p, x, M, y, di, dev)
                   : launch_tma<PACK, GS, ST, 1, OT, kXRmsNorm>(p, x, M, y, di, dev);
      if (p.prologue == W4A16_PROLOGUE_SWIGLU)
        return dec ? launch_tma<PACK, GS, ST, 1, OT, kXSwiGlu, false, kGeoDecode>(p, x, M, y, di, dev)
                   : launch_tma<PACK, GS, ST, 1, OT, kXSwiGlu>(p, x, M, y, di, dev);
      return dec ? launch_tma<PACK, GS, ST, 1, OT, kXCopy, false, kGeoDecode>(p, x, M, y, di, dev)
                 : launch_tma<PACK, GS, ST, 1, OT, kXCopy>(p, x, M, y, di, dev);
    }
    set_error("the staged (fused) GEMV takes the interleaved packing");
    return W4A16_ERR_DTYPE;
  }
  if (M == 1) {
    // one activation vector: keep it in shared memory when it fits beside the ring
    if constexpr (PACK == W4A16_PACK_INTERLEAVED) {
      if (p.tp_n > 1) {
        if (xs_fits) return launch_tma<PACK, GS, ST, 1, OT, kXCopy, true>(p, x, M, y, di, dev);
        return launch_tma<PACK, GS, ST, 1, OT, kXGlobal, true>(p, x, M, y, di, dev);
      }
    }
    if (xs_fits) return launch_tma<PACK, GS, ST, 1, OT, kXCopy>(p, x, M, y, di, dev);
    if (tma_smem_bytes<GS, ST, kGeoLong>() + tail_smem_bytes<PACK, 1, kXCopy>(p.K) <= di.smem_optin &&
        p.K <= kStageChunks * 8 * Geometry<kGeoLong>::kW * 32)
      return launch_tma<PACK, GS, ST, 1, OT, kXCopy, false, kGeoLong>(p, x, M, y, di, dev);
    return launch_tma<PACK, GS, ST, 1, OT, kXGlobal>(p, x, M, y, di, dev);
  }
  if (M <= 8) return launch_tma<PACK, GS, ST, 8, OT, kXGlobal>(p, x, M, y, di, dev);
  // many 32-row tiles (at least three per SM for every warp pair): the wide geometry
  if ((long long)(p.N + 2 * kMmaRows - 1) / (2 * kMmaRows) >= 3LL * di.sms)
    return launch_tma<PACK, GS, ST, 16, OT, kXGlobal, false, kGeoWide>(p, x, M, y, di, dev);
  return launch_tma<PACK, GS, ST, 16, OT, kXGlobal>(p, x, M, y, di, dev);
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

int current_sm_count(int* sms) {
  DeviceInfo di;
  const int rc = current_device_info(&di, nullptr);
  if (rc == W4A16_OK) *sms = di.sms;
  return rc;
}

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
  return kCounterBytes + (size_t)kMaxWarps * 2 * mc * kMaxTileRows * 4;
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
