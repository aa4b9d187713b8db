// W4A16 GEMM for many activation rows (prefill), sm_100a tensor cores (tcgen05, TMEM).
//
//   y[m, n] = sum_k x[m, k] * w16[n, k] (+ bias[n]),   w16 = fp16(fp32(q[n, k]) * scale(n, k))
//
// w16 is the reference's dequantised weight exactly (`dequant_int4`, the fp16 weight a
// caller without the dense copy multiplies by; the reference itself runs every call with
// more than one activation row through F.linear on fp16 weights, src/w4a16/kernels.py:
// 120-121).  The int4 codes are decoded into tensor memory, never into HBM: HBM carries
// N*K/2 packed bytes + scales + M*K*2 activation bytes + the output, against 2*N*K more
// written and read again by dequantise-then-GEMM.
//
// One CTA computes a 128 (weight rows) x BN (activation rows) tile over all of K:
//   warp 0       TMA copies per 64-column stage: the activation tile (BN x 64 fp16, 128-byte
//                swizzle: the tensor core's K-major canonical layout) and the packed weight
//                tile (128 rows x 32 bytes);
//   warp 1       allocates the 512 TMEM columns (the fp32 accumulator, then one decoded weight
//                tile per stage); one lane issues 4 tcgen05.mma per stage (M=128, N=BN, K=16,
//                A = decoded weights from TMEM, B = activations from shared memory, fp32 sums
//                in TMEM) and commits each stage's completion to the stage's "empty" barrier,
//                the last one to the accumulator barrier;
//   warps 2..    G decoder groups of four warps (G = 3 for BN = 256, 4 for 128); group g decodes
//                stages g, g+G, g+2G, ..., so G stages are decoded at once (one warp's pass over
//                a stage is latency-bound: barrier test, decode, TMEM store, arrive).  Thread r of
//                a group owns weight row r: it reads the row's 8 packed words of the stage, forms
//                w16 (exact codes, one fp32 multiply, one rounding to fp16 as the reference's
//                dequantisation does) and stores the row's 64 weights into its own TMEM lane
//                (tcgen05.st: the weight tile never touches shared memory, whose bandwidth the
//                activation copies and MMA reads already use); scales are fetched one stage of
//                the group ahead.  Then the epilogue: the thread holds TMEM lane r (its warp's
//                lane quarter), reads its group's share of the row's BN accumulators (16-column
//                chunks dealt round-robin) with tcgen05.ld, adds the bias and stores y[m, n] (32
//                consecutive n per warp store).
// BN is 256 when that still gives every SM a tile, else 128.
// Every barrier wait is bounded (2 s of %globaltimer); a wait that gives up records error 5
// (w4a16_read_device_error), the CTA stops issuing work, waits (bounded) for the copies and
// MMAs it has in flight and frees its TMEM.  No cluster, no multicast, no peer memory.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "w4a16_device.cuh"
#include "w4a16_internal.h"

namespace w4a16 {

namespace {

constexpr int kGmRows = 128;     // weight rows per tile: the MMA's M, TMEM lanes
constexpr int kGmK = 64;         // columns per stage: one 128-byte swizzle atom of fp16
template <int BN>
constexpr int gm_stages() { return BN == 128 ? 8 : 6; }  // as deep as shared memory and TMEM allow
// Decoder groups (stages decoded at once; a group is one warp per TMEM lane quarter).  The
// stage count is a multiple of the group count, so every ring slot is always decoded by the
// same group, in order: a group never waits on a slot's next phase before it has seen the
// current one complete (a parity wait that ran a phase ahead would pass on the one before).
template <int BN>
constexpr int gm_groups() { return BN == 128 ? 4 : 3; }
template <int BN>
constexpr int gm_warps() { return 2 + 4 * gm_groups<BN>(); }  // 0: copies, 1: TMEM + MMA, rest: decode + epilogue
constexpr int kGmErrWait = 5;    // a pipeline wait gave up
constexpr uint64_t kGmWaitNs = 2000000000ull;

__device__ int g_gemm_error = 0;

__device__ __forceinline__ void gm_fail() { atomicCAS(&g_gemm_error, 0, kGmErrWait); }

template <int BN>
struct GmLayout {
  static constexpr int kStages = gm_stages<BN>();
  static_assert(kStages % gm_groups<BN>() == 0, "each ring slot belongs to one decoder group");
  static constexpr uint32_t kB = BN * kGmK * 2;       // activations, fp16
  static constexpr uint32_t kP = kGmRows * kGmK / 2;  // packed weights
  static constexpr uint32_t kStage = kB + kP;
  static_assert(kB % 1024 == 0, "swizzled tiles start on 1024-byte boundaries");
  static_assert(kStage % 1024 == 0, "stages start on 1024-byte boundaries");
  // TMEM columns: the fp32 accumulator [0, BN), then per stage the decoded weight tile
  // (128 lanes = rows, 64 fp16 = 32 columns of two each)
  static constexpr uint32_t kTmemA = BN;
  static constexpr uint32_t kTmemCols = 512;
  static_assert(kTmemA + kStages * (kGmK / 2) <= kTmemCols, "accumulator and weight stages fit TMEM");
  // [1024 alignment slack][stages][full, decoded, empty barriers per stage, accumulator
  // barrier, TMEM address]
  static constexpr uint32_t kBarOff = kStages * kStage;
  static constexpr uint32_t kBytes = 1024 + kBarOff + (3 * kStages + 1) * 8 + 8;
  static_assert(kBytes <= 232448, "fits the 227 KB of shared memory a CTA may use");
};

// K-major operand tile with the 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes
// apart (stride byte offset), the leading byte offset unused by this layout (1), descriptor
// version 1, layout type 2 (SWIZZLE_128B).  Advancing K by 16 elements inside the atom adds
// 32 bytes to the start address.
__device__ __forceinline__ uint64_t gm_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: D fp32, A and B fp16, both K-major, N = BN, M = 128.
template <int BN>
__device__ __forceinline__ uint32_t gm_idesc() {
  return (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kGmRows >> 4) << 24);
}

// D (+)= A * B^T with A in tensor memory (K-major: lane = row, two fp16 per 32-bit column) and B
// in shared memory (gm_desc).
__device__ __forceinline__ void gm_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane, written and waited for.
__device__ __forceinline__ void gm_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, "
      "%31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
      "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void gm_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void gm_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void gm_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// 16 consecutive fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void gm_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

struct GemmParams {
  const float* scale;  // [N] or [N][K/128]
  const float* bias;   // [N] or null
  void* y;             // [M][N] fp32 or fp16
  int M, N, K, group;
  // split K (gridDim.z splits of kb_per_split stages): per-tile arrival counters and fp32
  // partial tiles [tile][split][BN columns][128 lanes] in the caller's workspace
  unsigned* cnt;
  float* part;
  int kb_per_split;
};

template <int BN, typename OT>
__global__ void __launch_bounds__(gm_warps<BN>() * 32, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap pmap,
              const GemmParams p) {
  using L = GmLayout<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  const uint32_t bars = base + L::kBarOff;
  auto full_bar = [&](int s) { return bars + (uint32_t)s * 8u; };
  auto dec_bar = [&](int s) { return bars + (uint32_t)(L::kStages + s) * 8u; };
  auto empty_bar = [&](int s) { return bars + (uint32_t)(2 * L::kStages + s) * 8u; };
  const uint32_t acc_bar = bars + 3u * L::kStages * 8u;
  const uint32_t tmem_slot = acc_bar + 8u;
  auto stage_b = [&](int s) { return base + (uint32_t)s * L::kStage; };
  auto stage_p = [&](int s) { return stage_b(s) + L::kB; };
  auto tmem_a = [&](uint32_t tmem, int s) { return tmem + L::kTmemA + (uint32_t)s * (kGmK / 2); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kGmRows;
  const int m0 = blockIdx.y * BN;
  // this CTA's stages: [kb0, kb0 + nk) of the K / 64 (all of them without a split)
  const int splits = gridDim.z;
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int nk_all = p.K / kGmK;
  const int nk = (kb0 + p.kb_per_split < nk_all ? p.kb_per_split : nk_all - kb0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(dec_bar(s), 4);  // the four warps of the group that decodes the stage
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(acc_bar, 1);
    mbar_fence_init();
    tma_prefetch_desc(&xmap);
    tma_prefetch_desc(&pmap);
  }
  if (warp == 1) {  // the whole warp allocates TMEM, then gives up the right to allocate more
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                 "r"(L::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  gm_fence_before();
  __syncthreads();
  gm_fence_after();
  uint32_t tmem_d;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(tmem_d) : "r"(tmem_slot) : "memory");

  if (warp == 0) {
    if (lane == 0) {  // copies
      const uint64_t keep = 0, stream_once = l2_policy_evict_first();
      (void)keep;
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < nk; ++i) {  // i: this CTA's stage count, kb: the column block
        const int kb = kb0 + i, s = i % L::kStages, u = i / L::kStages;
        if (u > 0 && !mbar_wait_bounded(empty_bar(s), (u - 1) & 1, kGmWaitNs)) {
          gm_fail();
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(full_bar(s), L::kB + L::kP);
        // activations are re-read by every weight-row tile: default L2 policy
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
            "[%0], [%1, {%2, %3}], [%4];" ::"r"(stage_b(s)),
            "l"(reinterpret_cast<uint64_t>(&xmap)), "r"(kb * kGmK), "r"(m0), "r"(full_bar(s))
            : "memory");
        tma_load_2d(stage_p(s), &pmap, kb * (kGmK / 2), n0, full_bar(s), stream_once);
        ++issued;
      }
      // the copies this thread issued have all landed before the CTA can exit
      for (int i = issued - L::kStages < 0 ? 0 : issued - L::kStages; i < issued; ++i)
        if (!mbar_wait_bounded(full_bar(i % L::kStages), (i / L::kStages) & 1, kGmWaitNs)) gm_fail();
      (void)ok;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issue
      const uint32_t idesc = gm_idesc<BN>();
      for (int i = 0; i < nk; ++i) {
        const int s = i % L::kStages, u = i / L::kStages;
        if (!mbar_wait_bounded(full_bar(s), u & 1, kGmWaitNs) ||
            !mbar_wait_bounded(dec_bar(s), u & 1, kGmWaitNs)) {
          gm_fail();
          break;
        }
        gm_fence_after();
        const uint32_t ta = tmem_a(tmem_d, s);
        const uint64_t db = gm_desc(stage_b(s));
#pragma unroll
        for (int kk = 0; kk < kGmK / 16; ++kk)  // K += 16: +8 TMEM columns of A, +32 bytes of B
          gm_mma_ts(tmem_d, ta + 8u * kk, db + 2u * kk, idesc, (i | kk) != 0);
        gm_commit(empty_bar(s));
      }
      gm_commit(acc_bar);  // every MMA issued above (or none) is complete when this arrives
    }
  } else {
    // decode, then epilogue.  Decoder group g (warps 2 + 4g .. 5 + 4g, one per TMEM lane
    // quarter) decodes the stages kb = g, g + G, g + 2G, ...: G stages are decoded at once,
    // since one warp's pass over a stage is latency-bound.  Thread r (0..127) of a group owns
    // weight row r (all 8 packed words of the stage) and, in the epilogue, the 16-column
    // accumulator chunks g, g + G, ... of TMEM lane r.
    constexpr int kG = gm_groups<BN>();
    const int quarter = warp & 3;
    const int grp = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const int n = n0 + r;
    const bool row_in = n < p.N;
    const int ng = p.group ? p.K / p.group : 1;
    const int kb_per_group = p.group ? p.group / kGmK : nk_all;  // column blocks sharing one scale
    auto scale_of = [&](int kb) {  // kb: column block of the whole K
      return row_in ? __ldg(p.scale + (size_t)n * ng + kb / kb_per_group) : 0.f;
    };
    // this group's first stage's scale, and its next stage's already on its way
    float sc = grp < nk ? scale_of(kb0 + grp) : 0.f;
    float sc_next = grp + kG < nk ? scale_of(kb0 + grp + kG) : 0.f;
    bool ok = true;
    for (int i = grp; i < nk; i += kG) {
      const int s = i % L::kStages, u = i / L::kStages;
      if (i != grp) {
        sc = sc_next;
        sc_next = i + kG < nk ? scale_of(kb0 + i + kG) : 0.f;
      }
      // the decision to stop is warp-uniform: __syncwarp and tcgen05.ld need every lane
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(full_bar(s), u & 1, kGmWaitNs))) {
        if (lane == 0) gm_fail();
        ok = false;
        break;
      }
      const uint4 w0 = lds128(stage_p(s) + (uint32_t)r * 32u);
      const uint4 w1 = lds128(stage_p(s) + (uint32_t)r * 32u + 16u);
      const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      uint32_t hv[32];  // row r's 64 weights of the stage, two fp16 per TMEM column
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // word j: columns 8j..8j+7 of the stage (interleaved packing)
        uint32_t o[4];
        decode_word(words[j], o);  // exact codes, pairs (0,1) (2,3) (4,5) (6,7)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&o[i]));
          // one packed conversion (round to nearest per element, as two separate ones would)
          const __half2 w2 = __floats2half2_rn(__fmul_rn(f.x, sc), __fmul_rn(f.y, sc));
          hv[4 * j + i] = *reinterpret_cast<const uint32_t*>(&w2);
        }
      }
      // into this thread's TMEM lane; complete before the stage is announced
      gm_st32(tmem_a(tmem_d, s) + ((uint32_t)(quarter * 32) << 16), hv);
      gm_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dec_bar(s));
    }
    // epilogue
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(acc_bar, 0, kGmWaitNs))) {
      if (lane == 0) gm_fail();
      ok = false;
    }
    gm_fence_after();
    if (ok && splits == 1) {
      const float b = (p.bias && row_in) ? __ldg(p.bias + n) : 0.f;
      OT* y = static_cast<OT*>(p.y);
      // 16-column chunks of the accumulator dealt round-robin to the groups
#pragma unroll 1
      for (int c0 = grp * 16; c0 < BN; c0 += 16 * kG) {
        float v[16];
        gm_ld16(tmem_d + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, v);
        if (row_in) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int m = m0 + c0 + i;
            if (m < p.M) y[(size_t)m * p.N + n] = from_f32<OT>(v[i] + b);
          }
        }
      }
    } else if (ok) {  // split K: this split's partial tile, column by column over the 128 lanes
      float* part = p.part + ((size_t)(blockIdx.y * gridDim.x + blockIdx.x) * splits + blockIdx.z) *
                                 (size_t)(BN * kGmRows);
#pragma unroll 1
      for (int c0 = grp * 16; c0 < BN; c0 += 16 * kG) {
        float v[16];
        gm_ld16(tmem_d + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) __stcg(part + (size_t)(c0 + i) * kGmRows + r, v[i]);
      }
      __threadfence();
    }
  }
  gm_fence_before();
  __syncthreads();
  if (splits > 1) {
    // The last split to finish a tile sums the partials in split order (the same order
    // whichever arrives last: deterministic), adds the bias, writes y and re-arms the counter.
    const uint32_t last_slot = tmem_slot + 4u;
    unsigned* cnt = p.cnt + (blockIdx.y * gridDim.x + blockIdx.x);
    if (threadIdx.x == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(cnt, 1u);
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(last_slot), "r"((unsigned)(prev == (unsigned)splits - 1u))
                   : "memory");
    }
    __syncthreads();
    unsigned last;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(last) : "r"(last_slot) : "memory");
    if (last) {
      __threadfence();
      const float* part = p.part + (size_t)(blockIdx.y * gridDim.x + blockIdx.x) * splits * (size_t)(BN * kGmRows);
      OT* y = static_cast<OT*>(p.y);
      // float4 pieces (4 lanes of one column), 4 pieces per thread in flight at once
      constexpr int kVec = BN * kGmRows / 4;
      const float4* part4 = reinterpret_cast<const float4*>(part);
      for (int base = threadIdx.x; base < kVec; base += 4 * blockDim.x) {
        float4 acc[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int sp = 0; sp < splits; ++sp) {  // split order: the same sum whichever CTA is last
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int e4 = base + u * blockDim.x;
            if (e4 < kVec) {
              const float4 v = __ldcg(part4 + (size_t)sp * kVec + e4);
              acc[u].x += v.x;
              acc[u].y += v.y;
              acc[u].z += v.z;
              acc[u].w += v.w;
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e4 = base + u * blockDim.x;
          if (e4 >= kVec) continue;
          const int c = (e4 * 4) / kGmRows, rr = (e4 * 4) % kGmRows, m = m0 + c;
          if (m >= p.M) continue;
          const float a4[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int nn = n0 + rr + j;
            if (nn < p.N) y[(size_t)m * p.N + nn] = from_f32<OT>(a4[j] + (p.bias ? __ldg(p.bias + nn) : 0.f));
          }
        }
      }
      if (threadIdx.x == 0) *cnt = 0u;
    }
  }
  if (warp == 1) {
    gm_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d),
                 "r"(L::kTmemCols)
                 : "memory");
  }
}

typedef CUresult (*GmEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                               const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                               const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                               CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

GmEncodeFn gm_encode_fn() {
  static GmEncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GmEncodeFn>(ptr);
  });
  return fn;
}

template <int BN, typename OT>
int launch_gemm_bn(const uint8_t* packed, const void* x, const GemmParams& prm, cudaStream_t stream) {
  using L = GmLayout<BN>;
  static std::atomic<uint64_t> configured{0};  // one bit per device
  int dev = 0;
  cudaError_t ae = cudaGetDevice(&dev);
  if (ae == cudaSuccess && dev < 64 && !(configured.load(std::memory_order_acquire) >> dev & 1ull)) {
    ae = cudaFuncSetAttribute(k_gemm_tc<BN, OT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)L::kBytes);
    if (ae == cudaSuccess) configured.fetch_or(1ull << dev, std::memory_order_acq_rel);
  }
  if (ae != cudaSuccess || dev >= 64) {
    set_error("configuring k_gemm_tc (%u bytes of shared memory): %s", L::kBytes,
              ae != cudaSuccess ? cudaGetErrorString(ae) : "device index out of range");
    return W4A16_ERR_CUDA;
  }
  GmEncodeFn enc = gm_encode_fn();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled entry point unavailable");
    return W4A16_ERR_CUDA;
  }
  CUtensorMap xmap, pmap;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)prm.K, (cuuint64_t)prm.M};
    const cuuint64_t strides[1] = {(cuuint64_t)prm.K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kGmK, (cuuint32_t)BN};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled(activations) failed: %d", (int)r);
      return W4A16_ERR_CUDA;
    }
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)(prm.K / 2), (cuuint64_t)prm.N};
    const cuuint64_t strides[1] = {(cuuint64_t)(prm.K / 2)};
    const cuuint32_t box[2] = {(cuuint32_t)(kGmK / 2), (cuuint32_t)kGmRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&pmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(packed), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled(packed weights) failed: %d", (int)r);
      return W4A16_ERR_CUDA;
    }
  }
  const int nk = prm.K / kGmK;
  const dim3 grid((prm.N + kGmRows - 1) / kGmRows, (prm.M + BN - 1) / BN,
                  (nk + prm.kb_per_split - 1) / prm.kb_per_split);
  k_gemm_tc<BN, OT><<<grid, gm_warps<BN>() * 32, L::kBytes, stream>>>(xmap, pmap, prm);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("k_gemm_tc launch failed: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  return W4A16_OK;
}

// How a call is cut up: 256 activation rows per tile when that still gives every SM a tile
// (half the decode work per flop), else 128; and when even 128-row tiles leave SMs idle, K
// is split across CTAs (at most 8 splits of at least 8 stages each), the splits' partial
// tiles summed by the last one to finish.
struct GemmPlan {
  bool wide = false;
  int splits = 1, kb_per_split = 0;
  size_t workspace = 0;  // bytes: counters (256-byte block) + partial tiles
};

GemmPlan gemm_plan(int M, int N, int K, int sms) {
  GemmPlan g;
  const int nk = K / kGmK, ntn = (N + kGmRows - 1) / kGmRows;
  const long long tiles256 = (long long)ntn * ((M + 255) / 256);
  const long long tiles128 = (long long)ntn * ((M + 127) / 128);
  g.wide = M > 128 && tiles256 >= sms;
  g.kb_per_split = nk;
  if (!g.wide && tiles128 < sms) {
    int s = (int)(sms / tiles128);
    if (s > 8) s = 8;
    if (s > nk / 8) s = nk / 8;
    if (s >= 2) {
      g.kb_per_split = (nk + s - 1) / s;
      g.splits = (nk + g.kb_per_split - 1) / g.kb_per_split;
    }
  }
  if (g.splits > 1) {
    const size_t cnt = ((size_t)tiles128 * 4 + 255) & ~(size_t)255;
    g.workspace = cnt + (size_t)tiles128 * g.splits * 128 * kGmRows * 4;
  }
  return g;
}

}  // namespace

size_t gemm_workspace_bytes(int M, int N, int K) {
  int sms = 0;
  if (M <= 0 || N <= 0 || K < kGmK || current_sm_count(&sms) != W4A16_OK) return 0;
  return gemm_plan(M, N, K, sms).workspace;
}

int launch_gemm(const uint8_t* packed, const float* scale, int group, const void* x, const float* bias,
                int M, int N, int K, void* y, int out_dtype, void* workspace, size_t workspace_bytes,
                cudaStream_t stream) {
  GemmParams prm;
  prm.scale = scale;
  prm.bias = bias;
  prm.y = y;
  prm.M = M;
  prm.N = N;
  prm.K = K;
  prm.group = group;
  prm.cnt = nullptr;
  prm.part = nullptr;
  int sms = 0;
  const int rc = current_sm_count(&sms);
  if (rc != W4A16_OK) return rc;
  GemmPlan g = gemm_plan(M, N, K, sms);
  if (g.splits > 1 && (!workspace || workspace_bytes < g.workspace)) {  // no room: no split
    g.splits = 1;
    g.kb_per_split = K / kGmK;
  }
  prm.kb_per_split = g.kb_per_split;
  if (g.splits > 1) {
    const int ntn = (N + kGmRows - 1) / kGmRows, tiles = ntn * ((M + 127) / 128);
    prm.cnt = static_cast<unsigned*>(workspace);
    prm.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + (((size_t)tiles * 4 + 255) & ~(size_t)255));
  }
  if (out_dtype == W4A16_DTYPE_F32)
    return g.wide ? launch_gemm_bn<256, float>(packed, x, prm, stream)
                  : launch_gemm_bn<128, float>(packed, x, prm, stream);
  return g.wide ? launch_gemm_bn<256, __half>(packed, x, prm, stream)
                : launch_gemm_bn<128, __half>(packed, x, prm, stream);
}

int read_gemm_error(int* code, cudaStream_t stream) {
  int h = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_gemm_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess && h != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_gemm_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  }
  if (e != cudaSuccess) {
    set_error("reading the GEMM error word: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  *code = h;
  return W4A16_OK;
}

}  // namespace w4a16
