// Shared pieces of the sm_100a W4A16 GEMV kernels (k_gemv_tma in w4a16_gemv.cu and the
// persistent decode-step kernel in w4a16_decode_step.cu): the shared-memory layout of a
// TMA-filled weight stage, the staged-activation layout, and the consumption of one
// stage (decode in registers, tensor-core dot product, group scales).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "w4a16_b200.h"
#include "w4a16_device.cuh"

#ifndef W4A16_FOLD  // batch-1 decode with half the nibbles left biased (decode_word_fold)
#define W4A16_FOLD 1
#endif
#ifndef W4A16_FOLD_LO  // group-128 batch-1 decode with every nibble left biased (decode_word_fold_all)
#define W4A16_FOLD_LO 0
#endif
#ifndef W4A16_ROW_NORESET  // per-row batch-1: one accumulation per tile, bias removed once per window
#define W4A16_ROW_NORESET 1
#endif

namespace w4a16 {

constexpr int kMmaRows = 16;      // rows of one m16n8k16 A fragment
constexpr int kSlabCols = 256;    // columns per 128-byte slab of a packed row

// Shared-memory stage of one warp: a window of SLABS 256-column slabs of RT*16 rows,
// one 3-D TMA box laid out [row][slab][128 B] with the 128-byte swizzle (1024-byte
// aligned), so every row of the box is one 512-byte run of global memory; and, for
// group-128, the window's scale tile [row][2*SLABS].
template <int SLABS, int RT, int GS, typename ST>
struct StageLayout {
  static_assert(SLABS == 4, "the swizzled [row][slab] layout is bank-conflict free for 4 slabs");
  static constexpr int kRows = kMmaRows * RT;
  static constexpr int kWBytes = kRows * SLABS * 128;
  static constexpr int kWStride = (kWBytes + 1023) / 1024 * 1024;
  static constexpr int kGroups = SLABS * 2;  // 128-column groups per window
  static constexpr int kSBytes = GS ? kRows * kGroups * (int)sizeof(ST) : 0;
  static constexpr int kSStride = (kSBytes + 127) / 128 * 128;
  static constexpr bool kScaleBoxOk = !GS || (kGroups * sizeof(ST)) % 16 == 0;
};

// Shared-memory plan of one CTA (offsets from the 1024-byte aligned base):
//   [W rings: WARPS x STAGES x kWStride][scale rings: WARPS x STAGES x kSStride]
//   [mbarriers: WARPS x STAGES x 8][staged activation at a 128-byte boundary]
template <int WARPS, int STAGES, typename L>
struct SmemPlan {
  static constexpr int kScaleOff = WARPS * STAGES * L::kWStride;
  static constexpr int kBarOff = kScaleOff + WARPS * STAGES * L::kSStride;
  static constexpr int kXOff = (kBarOff + WARPS * STAGES * 8 + 127) / 128 * 128;
  // dynamic bytes requested: the plan plus slack for aligning the base to 1024
  static constexpr int kBytes = kXOff + 1024;
  static_assert(kScaleOff % 1024 == 0 && kBarOff % 16 == 0 && kXOff % 128 == 0, "smem alignment");
};

// Byte offset of logical 16-byte chunk c of (row r, slab sl) inside a stage.  The
// 128-byte swizzle puts chunk c of 128-byte smem line L at c ^ (L & 7), L = 4r + sl:
// rows g and g+8 of one MMA get the same XOR, and the two rows a quarter-warp reads
// (g even and odd) get XORs that differ in bit 2, so its 8 lanes hit 8 bank groups.
template <int SLABS>
__device__ __forceinline__ uint32_t w_offset(int r, int sl, int c) {
  const int line = r * SLABS + sl;
  return (uint32_t)(line * 128 + ((c ^ (line & 7)) << 4));
}

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

// One window of one warp: slabs [sl_first, nslab) (all SLABS when FULL) of RT*16 rows.
// Shared-memory copy of a single activation vector, ordered so that the B fragment
// of (128-column group G, chunk j, thread t) is 16 bytes at ((G*4 + j)*4 + t)*16: the
// four threads of a group read 64 contiguous bytes, one conflict-free wavefront.
__device__ __forceinline__ uint32_t xs_offset(int col) {
  const int grp = col >> 7, off = col & 127;
  return (uint32_t)(((grp * 4 + ((off & 31) >> 3)) * 4 + (off >> 5)) * 16);
}

// Lane part of the weight-fragment offsets: for chunk c = gh*4 + t of slab sl in row
// r = g (row g + 8 adds 8 lines = 4096 bytes, rt adds 16 rows), the swizzled offset
// w_offset<4>(g, sl, c) depends only on the lane and (gh, sl): computed once.
struct LaneOffsets {
  uint32_t w[2][4];  // [gh][sl]
  uint32_t x;        // t * 16 (fragment order of the staged activation)
};

__device__ __forceinline__ LaneOffsets lane_offsets(int g, int t) {
  LaneOffsets o;
#pragma unroll
  for (int gh = 0; gh < 2; ++gh)
#pragma unroll
    for (int sl = 0; sl < 4; ++sl) o.w[gh][sl] = w_offset<4>(g, sl, gh * 4 + t);
  o.x = (uint32_t)t * 16u;
  return o;
}

// FOLD (one activation vector): weights decoded with
// decode_word_fold (or, with FOLD_LO, decode_word_fold_all), leaving a known bias on
// the codes; corr[group] = -(bias x sum of x over the group's biased columns) cancels it
// exactly up to fp32 rounding.
//   group-128: every group's accumulation starts from C = 0 and its sum enters tot as
//              scale * (acc + corr[group]);
//   per-row (ROWFOLD): one accumulation runs over the whole tile segment, and the
//              window's correction (the sum of its groups' corr) is added once per
//              window in the epilogue; the bias of one row stays a few thousand at
//              most, where fp32 keeps ~1e-4 absolute.
template <bool FULL, bool XS, int PACK, int GS, typename ST, int NB, int RT, int SLABS, bool FOLD,
          bool FOLDLO>
__device__ __forceinline__ void consume_window(uint32_t wbase, uint32_t sbase, uint32_t xs,
                                               uint32_t corr, int nslab, int kcol0,
                                               const __half* xg, int xk, int xm, int g, int t,
                                               const LaneOffsets& lo,
                                               float (&acc)[RT][2][BatchCfg<NB>::kHalves][4],
                                               float (&tot)[RT][BatchCfg<NB>::kHalves][4],
                                               int sl_first = 0) {
  // activation fragments of this window: 16 bytes at xwin + ((sl*2 + gh)*4 + j)*64
  const uint32_t xwin = xs + lo.x + (uint32_t)(kcol0 >> 7) * 256u;
  constexpr int NH = BatchCfg<NB>::kHalves;
  constexpr int kGroups = SLABS * 2;
  constexpr bool ROWFOLD = FOLD && !GS && W4A16_ROW_NORESET;
  static_assert(!FOLD || NB == 1, "FOLD: one activation vector");
  static_assert(!FOLDLO || (FOLD && GS), "FOLDLO: group-128 folded decode only");
#pragma unroll
  for (int sl = 0; sl < SLABS; ++sl) {
    if (FULL || (sl >= sl_first && sl < nslab)) {  // slabs [sl_first, nslab) unless FULL
      const int kcol = kcol0 + sl * kSlabCols;
      float cinit[2] = {0.f, 0.f};
      if (FOLD && !ROWFOLD) {
#pragma unroll
        for (int gh = 0; gh < 2; ++gh) cinit[gh] = lds_f32(corr + (uint32_t)((kcol >> 7) + gh) * 4u);
      }
      uint4 wa[RT][2], wb[RT][2];
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int gh = 0; gh < 2; ++gh) {
          const int c = gh * 4 + t;
          (void)c;
          wa[rt][gh] = lds128(wbase + lo.w[gh][sl] + rt * 16 * SLABS * 128);
          wb[rt][gh] = lds128(wbase + lo.w[gh][sl] + rt * 16 * SLABS * 128 + 8 * SLABS * 128);
        }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int gh = 0; gh < 2; ++gh) {
          const int col = kcol + gh * 128 + 32 * t + 8 * j;
          uint4 xv[NH];
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            xv[h] = XS ? lds128(xwin + ((sl * 2 + gh) * 4 + j) * 64)
                       : load_x<NB>(xg, xk, xm, g, h, col);
            if (PACK == W4A16_PACK_SIMPLE && !XS) xv[h] = simple_order(xv[h]);  // staged pre-ordered
          }
#pragma unroll
          for (int rt = 0; rt < RT; ++rt) {
            const uint4& va = wa[rt][gh];
            const uint4& vb = wb[rt][gh];
            const uint32_t word_a = j == 0 ? va.x : j == 1 ? va.y : j == 2 ? va.z : va.w;
            const uint32_t word_b = j == 0 ? vb.x : j == 1 ? vb.y : j == 2 ? vb.z : vb.w;
            uint32_t A[4], B[4];
            if (FOLDLO) {
              decode_word_fold_all(word_a, A);
              decode_word_fold_all(word_b, B);
            } else if (FOLD) {
              decode_word_fold(word_a, A);
              decode_word_fold(word_b, B);
            } else {
              decode_word(word_a, A);
              decode_word(word_b, B);
            }
#pragma unroll
            for (int h = 0; h < NH; ++h) {
              if (GS && j == 0)  // every group-128 sum starts from zero
                mma_16816_zc(acc[rt][gh][h], A[0], B[0], A[1], B[1], xv[h].x, xv[h].y);
              else if (FOLD && !ROWFOLD && j == 0)
                mma_16816_c(acc[rt][gh][h], A[0], B[0], A[1], B[1], xv[h].x, xv[h].y, cinit[gh]);
              else
                mma_16816(acc[rt][gh][h], A[0], B[0], A[1], B[1], xv[h].x, xv[h].y);
              mma_16816(acc[rt][gh][h], A[2], B[2], A[3], B[3], xv[h].z, xv[h].w);
            }
          }
        }
      }
      if (GS) {
#pragma unroll
        for (int rt = 0; rt < RT; ++rt)
#pragma unroll
          for (int gh = 0; gh < 2; ++gh) {
            const int grp = sl * 2 + gh;
            const int ra = rt * 16 + g;
            float s0, s1;
            if (sizeof(ST) == 4) {
              s0 = lds_f32(sbase + (ra * kGroups + grp) * 4);
              s1 = lds_f32(sbase + ((ra + 8) * kGroups + grp) * 4);
            } else {
              s0 = __half2float(__ushort_as_half(lds_u16(sbase + (ra * kGroups + grp) * 2)));
              s1 = __half2float(__ushort_as_half(lds_u16(sbase + ((ra + 8) * kGroups + grp) * 2)));
            }
            // FOLD: the group's bias correction joins its sum before the scale
            const float cg = FOLD ? cinit[gh] : 0.f;
#pragma unroll
            for (int h = 0; h < NH; ++h) {
              // one activation vector: the MMA's columns are copies, only 0 and 2 are used
              tot[rt][h][0] = fmaf(s0, FOLD ? acc[rt][gh][h][0] + cg : acc[rt][gh][h][0], tot[rt][h][0]);
              if (NB != 1) tot[rt][h][1] = fmaf(s0, acc[rt][gh][h][1], tot[rt][h][1]);
              tot[rt][h][2] = fmaf(s1, FOLD ? acc[rt][gh][h][2] + cg : acc[rt][gh][h][2], tot[rt][h][2]);
              if (NB != 1) tot[rt][h][3] = fmaf(s1, acc[rt][gh][h][3], tot[rt][h][3]);
            }
          }
      } else if (FOLD && !ROWFOLD) {  // per-row scale: the groups are summed unscaled
#pragma unroll
        for (int rt = 0; rt < RT; ++rt)
#pragma unroll
          for (int gh = 0; gh < 2; ++gh)
#pragma unroll
            for (int h = 0; h < NH; ++h)
#pragma unroll
              for (int i = 0; i < 4; ++i) tot[rt][h][i] += acc[rt][gh][h][i];
      }
    }
  }
}

// Latency-oriented consume_window for one activation vector staged in shared memory,
// interleaved packing, group-128 scales of type ST and a full window (4 slabs): SPAN slabs
// at a time have their weights loaded first, then their 2 * SPAN 128-column groups
// accumulate as independent MMA chains interleaved step by step (k-chunk j outer), so a
// warp working alone on a window waits for about 8 * 4 / SPAN MMA latencies instead of 32.
// Same arithmetic as consume_window<..., FOLD = true> (biased high nibbles, -72 * sum(x)
// correction per group, group sums scaled in fp32), group by group; only rows g and g + 8
// (tot[0], tot[2]) are kept.
template <int SPAN, typename ST>
__device__ __forceinline__ void consume_window_wide(uint32_t wbase, uint32_t sbase, uint32_t xs, uint32_t corr,
                                                    int kcol0, int g, const LaneOffsets& lo, float (&tot)[4]) {
  static_assert(SPAN == 1 || SPAN == 2 || SPAN == 4, "slabs per pass");
  constexpr int kGroups = 8;  // 128-column groups of a window
  const uint32_t xwin = xs + lo.x + (uint32_t)(kcol0 >> 7) * 256u;
#pragma unroll
  for (int s0 = 0; s0 < 4; s0 += SPAN) {
    uint4 wa[SPAN][2], wb[SPAN][2];
#pragma unroll
    for (int i = 0; i < SPAN; ++i)
#pragma unroll
      for (int gh = 0; gh < 2; ++gh) {
        wa[i][gh] = lds128(wbase + lo.w[gh][s0 + i]);
        wb[i][gh] = lds128(wbase + lo.w[gh][s0 + i] + 8 * 4 * 128);
      }
    float acc[2 * SPAN][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int i = 0; i < SPAN; ++i) {
#pragma unroll
        for (int gh = 0; gh < 2; ++gh) {
          const int k = i * 2 + gh;            // chain within the pass
          const int grp = (s0 + i) * 2 + gh;   // group within the window
          const uint4 xv = lds128(xwin + (uint32_t)((grp * 4 + j) * 64));
          const uint4& va = wa[i][gh];
          const uint4& vb = wb[i][gh];
          const uint32_t word_a = j == 0 ? va.x : j == 1 ? va.y : j == 2 ? va.z : va.w;
          const uint32_t word_b = j == 0 ? vb.x : j == 1 ? vb.y : j == 2 ? vb.z : vb.w;
          uint32_t A[4], B[4];
          decode_word_fold(word_a, A);
          decode_word_fold(word_b, B);
          if (j == 0)
            mma_16816_zc(acc[k], A[0], B[0], A[1], B[1], xv.x, xv.y);
          else
            mma_16816(acc[k], A[0], B[0], A[1], B[1], xv.x, xv.y);
          mma_16816(acc[k], A[2], B[2], A[3], B[3], xv.z, xv.w);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 2 * SPAN; ++k) {
      const int grp = s0 * 2 + k;
      const float cg = lds_f32(corr + (uint32_t)((kcol0 >> 7) + grp) * 4u);
      float sa, sb;
      if (sizeof(ST) == 4) {
        sa = lds_f32(sbase + (g * kGroups + grp) * 4);
        sb = lds_f32(sbase + ((g + 8) * kGroups + grp) * 4);
      } else {
        sa = __half2float(__ushort_as_half(lds_u16(sbase + (g * kGroups + grp) * 2)));
        sb = __half2float(__ushort_as_half(lds_u16(sbase + ((g + 8) * kGroups + grp) * 2)));
      }
      tot[0] = fmaf(sa, acc[k][0] + cg, tot[0]);
      tot[2] = fmaf(sb, acc[k][2] + cg, tot[2]);
    }
  }
}

}  // namespace w4a16
