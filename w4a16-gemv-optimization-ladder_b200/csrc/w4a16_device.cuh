// Device-side building blocks for the sm_100a W4A16 kernels: inline-PTX wrappers
// for the int4 -> fp16 nibble decode, the m16n8k16 tensor-core step, shared-memory
// and read-only global loads, mbarriers and TMA (cp.async.bulk.tensor) copies.
//
// Packed weight formats (both produced by the Python packers of this package and
// by the reference's src/w4a16/kernels.py:64-91):
//   interleaved  nibble slot i (bits 4i..4i+3 of a little-endian u32 holding 8
//                consecutive columns) holds column {0,2,4,6,1,3,5,7}[i]; the
//                stored nibble is q + 8 (kernels.py:73-91).
//   simple       byte c of a row holds (q[2c]+8) << 4 | (q[2c+1]+8)
//                (kernels.py:64-70).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace w4a16 {

// fp16 bit patterns used by the exponent-trick decode.
//   0x6400 | n      == 1024 + n           (n in 0..15)
//   0x6400 | n << 4 == 1024 + 16 n
// (1024 + n) - 1032          == n - 8  exactly (one subtraction)
// (1024 + 16 n) * 1/16 - 72  == n - 8  exactly (one fused multiply-add)
constexpr uint32_t kExp16x2 = 0x64006400u;   // {1024, 1024}
constexpr uint32_t kLoMask = 0x000f000fu;    // nibble 0 of each 16-bit half
constexpr uint32_t kHiMask = 0x00f000f0u;    // nibble 1 of each 16-bit half
constexpr uint32_t k1032x2 = 0x64086408u;    // {1032, 1032}
constexpr uint32_t kSixteenth = 0x2c002c00u; // {1/16, 1/16}
constexpr uint32_t kMinus72x2 = 0xd480d480u; // {-72, -72}
constexpr uint32_t kExp64x2 = 0x54005400u;   // {64, 64}
// LUT operand of lop3 for (a & b) | c, built from the canonical inputs
// a = 0xF0, b = 0xCC, c = 0xAA.
constexpr uint32_t kLutAndOr = (0xF0 & 0xCC) | 0xAA;

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(r) : "r"(a), "r"(b), "r"(c), "n"(kLutAndOr));
  return r;
}

__device__ __forceinline__ uint32_t sub_f16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t fma_f16x2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint32_t mul_f16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Decode one packed word (8 int4 codes of one row) into four f16x2 registers
// holding the signed codes q in [-8, 7], exactly.  Nine instructions: one shift,
// four lop3, two f16x2 subtractions, two f16x2 FMAs.
//   o[0] = nibble slots (0,4)   o[1] = slots (1,5)
//   o[2] = slots (2,6)          o[3] = slots (3,7)
// For the interleaved packing these are the column pairs (0,1) (2,3) (4,5) (6,7).
// For the simple packing they are the column pairs (1,5) (0,4) (3,7) (2,6).
__device__ __forceinline__ void decode_word(uint32_t w, uint32_t (&o)[4]) {
  const uint32_t w8 = w >> 8;
  const uint32_t lo0 = lop3_and_or(w, kLoMask, kExp16x2);
  const uint32_t hi0 = lop3_and_or(w, kHiMask, kExp16x2);
  const uint32_t lo1 = lop3_and_or(w8, kLoMask, kExp16x2);
  const uint32_t hi1 = lop3_and_or(w8, kHiMask, kExp16x2);
  o[0] = sub_f16x2(lo0, k1032x2);
  o[1] = fma_f16x2(hi0, kSixteenth, kMinus72x2);
  o[2] = sub_f16x2(lo1, k1032x2);
  o[3] = fma_f16x2(hi1, kSixteenth, kMinus72x2);
}

// The same four f16x2 with nibble 1 of each byte pair left biased: o[1] and o[3]
// hold 64 + n = q + 72 exactly (nibble at mantissa bits 4-7 under exponent 64), so no
// f16x2 operation is spent on them.  Seven instructions: one shift, four lop3, two
// f16x2 subtractions.  The caller removes 72 * (sum of the activation over those
// columns: pairs (2,3) and (6,7) of every 8 for the interleaved packing) per group.
__device__ __forceinline__ void decode_word_fold(uint32_t w, uint32_t (&o)[4]) {
  const uint32_t w8 = w >> 8;
  o[0] = sub_f16x2(lop3_and_or(w, kLoMask, kExp16x2), k1032x2);
  o[1] = lop3_and_or(w, kHiMask, kExp64x2);
  o[2] = sub_f16x2(lop3_and_or(w8, kLoMask, kExp16x2), k1032x2);
  o[3] = lop3_and_or(w8, kHiMask, kExp64x2);
}

// Every nibble left biased: o[0] and o[2] hold 1024 + n = q + 1032, o[1] and o[3] hold
// 64 + n = q + 72, all exact.  Five instructions: one shift, four lop3.  The caller
// removes 1032 * (sum of x over columns 0,1,4,5 of every 8) + 72 * (sum over 2,3,6,7)
// per group (interleaved packing).
__device__ __forceinline__ void decode_word_fold_all(uint32_t w, uint32_t (&o)[4]) {
  const uint32_t w8 = w >> 8;
  o[0] = lop3_and_or(w, kLoMask, kExp16x2);
  o[1] = lop3_and_or(w, kHiMask, kExp64x2);
  o[2] = lop3_and_or(w8, kLoMask, kExp16x2);
  o[3] = lop3_and_or(w8, kHiMask, kExp64x2);
}

// Reorder an 8-column activation chunk (four f16x2: (x0,x1) (x2,x3) (x4,x5) (x6,x7))
// into the column pairs that decode_word produces for the simple packing:
// (x1,x5) (x0,x4) (x3,x7) (x2,x6).
__device__ __forceinline__ uint4 simple_order(uint4 v) {
  uint4 r;
  r.x = prmt(v.x, v.z, 0x7632u);
  r.y = prmt(v.x, v.z, 0x5410u);
  r.z = prmt(v.y, v.w, 0x7632u);
  r.w = prmt(v.y, v.w, 0x5410u);
  return r;
}

// D += A(16x16, f16, row) * B(16x8, f16, col), f32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A * B + c (every element of C = c): starts an accumulation at an offset.
__device__ __forceinline__ void mma_16816_c(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                            uint32_t a3, uint32_t b0, uint32_t b1, float c) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c));
}

// D = A * B (C = 0): starts a fresh accumulation without zeroed registers.
__device__ __forceinline__ void mma_16816_zc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ unsigned short lds_u16(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// Read-only 16-byte global load (activations: tiny, reused by every row).
__device__ __forceinline__ uint4 ldg128(const void* p) {
  uint4 v;
  asm("ld.global.nc.v4.b32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// 16-byte load through L2 only: for data that another kernel may have written while
// this one was already running (programmatic dependent launch), where the
// non-coherent path is not allowed.
__device__ __forceinline__ uint4 ldcg128(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// silu(g) * u = g / (1 + exp(-g)) * u with the fast exponential and division intrinsics
// (for g -> -inf the divisor overflows and the quotient is 0, silu's limit).
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

// Two floats rounded to fp16 (round to nearest even), packed low | high.
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  return (uint32_t)__half_as_ushort(__float2half_rn(lo)) |
         ((uint32_t)__half_as_ushort(__float2half_rn(hi)) << 16);
}

// Raw bits of a scale, loaded where the call stands (volatile: the compiler may not
// sink the load to the value's first use), for scales used much later.
template <typename T>
__device__ __forceinline__ uint32_t ld_scale_bits_now(const T* p);
template <>
__device__ __forceinline__ uint32_t ld_scale_bits_now<float>(const float* p) {
  uint32_t v;
  asm volatile("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
template <>
__device__ __forceinline__ uint32_t ld_scale_bits_now<__half>(const __half* p) {
  unsigned short v;
  asm volatile("ld.global.nc.b16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
template <typename T>
__device__ __forceinline__ float scale_from_bits(uint32_t b);
template <>
__device__ __forceinline__ float scale_from_bits<float>(uint32_t b) { return __uint_as_float(b); }
template <>
__device__ __forceinline__ float scale_from_bits<__half>(uint32_t b) {
  return __half2float(__ushort_as_half((unsigned short)b));
}

// ------------------------------------------------ flags shared with other GPUs
// Release store / acquire load at system scope, for flags that peer GPUs read or write
// through NVLink-mapped memory.
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ------------------------------------------------ programmatic dependent launch
// A kernel launched with programmatic stream serialisation may start while the
// previous kernel in the stream is still running.  grid_dependency_wait() returns once
// that kernel has completed and its memory is visible (at once for a normal launch);
// grid_launch_dependents() lets the next such kernel be scheduled.  Kernels here call
// the trigger only after their own wait, so at most two consecutive kernels overlap.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ----------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of an mbarrier, giving up after `limit_ns` of wall time.
// Returns false on timeout; the caller records the failure and returns.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// ---------------------------------------------------------------------- TMA

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor copy global -> shared, completion signalled on `bar`
// (complete_tx).  The source is always this GPU's own memory and every CTA fetches
// its own tiles, one copy per CTA.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes."
      "L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

// 3-D tiled bulk tensor copy global -> shared, one copy per CTA, as tma_load_2d.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes."
      "L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
      : "memory");
}

// Contiguous bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16),
// completion signalled on `bar` (complete_tx).  The source is this GPU's own memory.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Orders this thread's earlier generic-proxy accesses to shared memory before later
// async-proxy (TMA / bulk copy) writes to it.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

}  // namespace w4a16
