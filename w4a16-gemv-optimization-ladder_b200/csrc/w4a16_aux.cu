// Companion kernels of the W4A16 GEMV path (sm_100a):
//   k_h2f32           lossy variant: fp16 products summed in fp16 per packed word,
//                     bit-identical to the reference k_h2f32 (kernels/w4a16_kernels.cu:161-171)
//   k_fp16_gemv       dense fp16 GEMV, fp32 accumulation: the bandwidth baseline
//                     (reference k_fp16, kernels/w4a16_kernels.cu:174-180)
//   k_dequant         bit-exact fp16 dequantisation of packed codes
//                     (the reference's dequant formula, src/w4a16/kernels.py:94-101)
//   k_quantize_pack   symmetric int4 quantisation + packing in one pass
//                     (src/w4a16/kernels.py:47-60 then :64-91, done in torch there)
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "w4a16_device.cuh"
#include "w4a16_internal.h"

namespace w4a16 {

namespace {

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s launch failed: %s", what, cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  return W4A16_OK;
}

// Bit offset of column c (0..7) inside a packed word.
__device__ __forceinline__ int column_shift(int packing, int c) {
  if (packing == W4A16_PACK_INTERLEAVED) return 4 * ((c & 1) ? 4 + (c >> 1) : (c >> 1));
  return (c >> 1) * 8 + ((c & 1) ? 0 : 4);
}

}  // namespace

// ------------------------------------------------------------------ h2f32 (lossy)

// The reference's arithmetic, step for step: one warp per row, lane l takes packed
// words l, l+32, l+64, ... in that order.  Per word the four column pairs (2k, 2k+1)
// run two fp16 chains (mul then three fma on f16x2, each step rounded once: even
// columns 0,2,4,6 in one half, odd columns 1,3,5,7 in the other), the two chain sums
// are widened and added in fp32 and added to the lane's fp32 sum; each lane's sum is
// multiplied by the row scale and the 32 are reduced by the shuffle tree
// p += shfl_down(p, o), o = 16 .. 1.  Being the same operations on the same operands in
// the same order, the output is bit-identical to the reference's.
//
// The warp walks its rows grid-strided (a resident grid) as a stream of (row, chunk)
// steps, a chunk being kH2Depth words per lane; the next step's words (and, before a
// row's last chunk, its scale) are in flight while the current chunk is summed.  A chunk
// is full or not for the whole warp, so full chunks run without per-word guards.  The
// activation vector is staged once per CTA in shared memory with each half2 swapped, so
// a word's pair k decodes as (low nibble, high nibble) of byte k: columns (2k+1, 2k)
// against (x[2k+1], x[2k]).  Longer vectors are read through L1 and swapped in registers.
// Measured alternative: two rows per warp in the two f16x2 halves (fewer decode
// instructions per word) ran slower here, its 64 registers leaving too few warps to
// cover the shared-memory loads.
#ifndef W4A16_H2_DEPTH  // words in flight per lane per (row, chunk)
#define W4A16_H2_DEPTH 8
#endif
#ifndef W4A16_H2_CTAS  // resident CTAs of 8 warps per SM
#define W4A16_H2_CTAS 6
#endif
constexpr int kH2Warps = 8;
constexpr int kH2Depth = W4A16_H2_DEPTH;
constexpr int kH2MaxStagedCols = 16384;  // 32 KB of fp16 per CTA
constexpr int kH2CtasPerSm = W4A16_H2_CTAS;
constexpr uint32_t kH2NibbleMask = 0x00F0000Fu;  // low nibble -> low half, high nibble -> high half
constexpr uint32_t kH2Exponents = 0x54006400u;   // {1024 + n, 64 + n} (high nibble sits at bits 4-7)
constexpr uint32_t kH2Bias = 0x54806408u;        // {1032, 72}

__device__ __forceinline__ uint4 swap_halves(uint4 v) {
  return make_uint4(prmt(v.x, v.x, 0x1032u), prmt(v.y, v.y, 0x1032u), prmt(v.z, v.z, 0x1032u),
                    prmt(v.w, v.w, 0x1032u));
}

// f32(even-column chain) + f32(odd-column chain) of one packed word (simple packing:
// byte k = code[2k] << 4 | code[2k+1], codes biased by 8); xv holds the swapped pairs.
__device__ __forceinline__ float h2f32_word(uint32_t v, const uint4& xv) {
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k)  // byte k in bytes 0 and 2, then its two nibbles, minus 8
    w[k] = sub_f16x2(lop3_and_or(prmt(v, v, 0x0101u * k), kH2NibbleMask, kH2Exponents), kH2Bias);
  uint32_t t = mul_f16x2(w[0], xv.x);
  t = fma_f16x2(w[1], xv.y, t);
  t = fma_f16x2(w[2], xv.z, t);
  t = fma_f16x2(w[3], xv.w, t);
  // f32(even) + f32(odd), rounded once in fp32 (addition commutes, so this is the
  // reference's low + high).  sm_100's mixed-precision add widens its f16 operand exactly
  // on the FMA pipe; adding the odd half to +0 first is exact too (a -0 becomes +0,
  // which no later sum can tell apart, every lane sum starting from +0).
  float r;
  asm("{\n .reg .f16 lo, hi;\n mov.b32 {lo, hi}, %1;\n add.rn.f32.f16 %0, lo, 0f00000000;\n"
      " add.rn.f32.f16 %0, hi, %0;\n}"
      : "=&f"(r)
      : "r"(t));
  return r;
}

template <bool STAGED>
__global__ void __launch_bounds__(kH2Warps * 32, kH2CtasPerSm)
    k_h2f32(const uint8_t* __restrict__ packed, const float* __restrict__ scale,
            const __half* __restrict__ vec, float* __restrict__ out, int rows, int cols) {
  __shared__ __align__(16) uint4 xs[STAGED ? kH2MaxStagedCols / 8 : 1];
  const int words = cols >> 3;
  if (STAGED) {
    for (int w = threadIdx.x; w < words; w += blockDim.x) xs[w] = swap_halves(ldg128(vec + (size_t)w * 8));
    __syncthreads();
  }
  const int lane = threadIdx.x & 31;
  const int stride = gridDim.x * kH2Warps;
  constexpr int kChunkWords = 32 * kH2Depth;  // words of one row a warp loads per step
  const int nchunk = (words + kChunkWords - 1) / kChunkWords;
  auto full = [&](int ch) { return (ch + 1) * kChunkWords <= words; };
  auto load = [&](int row, int ch, uint32_t (&buf)[kH2Depth]) {
    if (row >= rows) return;
    const uint32_t* wr = reinterpret_cast<const uint32_t*>(packed + (size_t)row * (cols >> 1));
    const int g0 = ch * kChunkWords + lane;
    if (full(ch)) {
#pragma unroll
      for (int d = 0; d < kH2Depth; ++d) buf[d] = __ldg(wr + g0 + 32 * d);
    } else {
#pragma unroll
      for (int d = 0; d < kH2Depth; ++d) buf[d] = g0 + 32 * d < words ? __ldg(wr + g0 + 32 * d) : 0u;
    }
  };
  auto xword = [&](int g) { return STAGED ? xs[g] : swap_halves(ldg128(vec + (size_t)g * 8)); };
  int row = blockIdx.x * kH2Warps + (threadIdx.x >> 5), ch = 0;
  float p = 0.f;
  // one step: issue the next step's loads into nxt, sum cur into p, finish the row
  auto step = [&](uint32_t (&cur)[kH2Depth], uint32_t (&nxt)[kH2Depth]) {
    int nrow = row, nch = ch + 1;
    if (nch == nchunk) {
      nch = 0;
      nrow += stride;
    }
    load(nrow, nch, nxt);
    const float sc = nch == 0 ? __ldg(scale + row) : 0.f;  // in flight while the words are summed
    const int g0 = ch * kChunkWords + lane;
    if (full(ch)) {
#pragma unroll
      for (int d = 0; d < kH2Depth; ++d) p += h2f32_word(cur[d], xword(g0 + 32 * d));
    } else {
#pragma unroll
      for (int d = 0; d < kH2Depth; ++d)
        if (g0 + 32 * d < words) p += h2f32_word(cur[d], xword(g0 + 32 * d));
    }
    if (nch == 0) {
      p = __fmul_rn(p, sc);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) p += __shfl_down_sync(0xffffffffu, p, o);
      if (lane == 0) out[row] = p;
      p = 0.f;
    }
    row = nrow;
    ch = nch;
  };
  uint32_t a[kH2Depth], b[kH2Depth];
  load(row, ch, a);
  while (row < rows) {
    step(a, b);
    if (row >= rows) break;
    step(b, a);
  }
}

int launch_h2f32(const uint8_t* packed, const float* scale, const void* vec, float* out, int rows,
                 int cols, cudaStream_t stream) {
  int sms = 0;
  const int rc = current_sm_count(&sms);
  if (rc != W4A16_OK) return rc;
  const long long need = (rows + kH2Warps - 1) / kH2Warps;
  const int grid = (int)(need < (long long)sms * kH2CtasPerSm ? need : (long long)sms * kH2CtasPerSm);
  const __half* v = static_cast<const __half*>(vec);
  if (cols <= kH2MaxStagedCols)
    k_h2f32<true><<<grid, kH2Warps * 32, 0, stream>>>(packed, scale, v, out, rows, cols);
  else
    k_h2f32<false><<<grid, kH2Warps * 32, 0, stream>>>(packed, scale, v, out, rows, cols);
  return check_launch("k_h2f32");
}

// ------------------------------------------------------------------- dense fp16

// One warp per row; each lane streams 16-byte chunks (8 fp16) with four loads in
// flight and accumulates in fp32.
__global__ void __launch_bounds__(256)
    k_fp16_gemv(const __half* __restrict__ mat, const __half* __restrict__ vec,
                float* __restrict__ out, int rows, int cols) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __half* mr = mat + (size_t)row * cols;
  const int chunks = cols >> 3;
  float acc = 0.f;
  int c = lane;
  for (; c + 96 < chunks; c += 128) {
    uint4 m[4], v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) m[u] = ldg128(mr + (size_t)(c + 32 * u) * 8);
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = ldg128(vec + (size_t)(c + 32 * u) * 8);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t mm[4] = {m[u].x, m[u].y, m[u].z, m[u].w};
      const uint32_t vv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&mm[i]));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&vv[i]));
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
      }
    }
  }
  for (; c < chunks; c += 32) {
    const uint4 m = ldg128(mr + (size_t)c * 8);
    const uint4 v = ldg128(vec + (size_t)c * 8);
    const uint32_t mm[4] = {m.x, m.y, m.z, m.w};
    const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&mm[i]));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&vv[i]));
      acc = fmaf(a.x, b.x, acc);
      acc = fmaf(a.y, b.y, acc);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) out[row] = acc;
}

int launch_fp16_gemv(const void* mat, const void* vec, float* out, int rows, int cols,
                     cudaStream_t stream) {
  const int grid = (rows + 7) / 8;
  k_fp16_gemv<<<grid, 256, 0, stream>>>(static_cast<const __half*>(mat),
                                         static_cast<const __half*>(vec), out, rows, cols);
  return check_launch("k_fp16_gemv");
}

// ---------------------------------------------------------------------- dequant

// One thread per packed word: eight fp16 outputs, written as one 16-byte store.
template <typename ST>
__global__ void __launch_bounds__(256)
    k_dequant(const uint32_t* __restrict__ packed, int packing, const ST* __restrict__ scale,
              int group, int rows, int cols, __half* __restrict__ out) {
  const int wpr = cols >> 3;
  const size_t total = (size_t)rows * wpr;
  const int ngroups = group ? cols / group : 1;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int row = (int)(idx / wpr);
    const int w = (int)(idx % wpr);
    const uint32_t word = __ldg(packed + idx);
    const float s = group ? to_f32<ST>(__ldg(scale + (size_t)row * ngroups + (w * 8) / group))
                          : to_f32<ST>(__ldg(scale + row));
    uint32_t pair[4];
#pragma unroll
    for (int c = 0; c < 8; c += 2) {
      const int q0 = (int)((word >> column_shift(packing, c)) & 0xFu) - 8;
      const int q1 = (int)((word >> column_shift(packing, c + 1)) & 0xFu) - 8;
      const unsigned short h0 = __half_as_ushort(__float2half_rn(__fmul_rn((float)q0, s)));
      const unsigned short h1 = __half_as_ushort(__float2half_rn(__fmul_rn((float)q1, s)));
      pair[c >> 1] = (uint32_t)h0 | ((uint32_t)h1 << 16);
    }
    *reinterpret_cast<uint4*>(out + idx * 8) = make_uint4(pair[0], pair[1], pair[2], pair[3]);
  }
}

int launch_dequant(const uint8_t* packed, int packing, const void* scale, int scale_dtype,
                   int group, int rows, int cols, void* out, cudaStream_t stream) {
  const size_t total = (size_t)rows * (cols / 8);
  size_t blocks = (total + 255) / 256;
  if (blocks > 65535u * 16u) blocks = 65535u * 16u;
  const uint32_t* pw = reinterpret_cast<const uint32_t*>(packed);
  if (scale_dtype == W4A16_DTYPE_F32)
    k_dequant<float><<<(unsigned)blocks, 256, 0, stream>>>(
        pw, packing, static_cast<const float*>(scale), group, rows, cols, static_cast<__half*>(out));
  else
    k_dequant<__half><<<(unsigned)blocks, 256, 0, stream>>>(
        pw, packing, static_cast<const __half*>(scale), group, rows, cols,
        static_cast<__half*>(out));
  return check_launch("k_dequant");
}

// ------------------------------------------------------------- quantise + pack

// One warp per row.  The row is walked in 128-column chunks, each lane holding
// four consecutive columns; two neighbouring lanes form one packed word.
template <typename WT, typename ST>
__global__ void __launch_bounds__(256)
    k_quantize_pack(const WT* __restrict__ w, int rows, int cols, int group, int packing,
                    uint8_t* __restrict__ packed, ST* __restrict__ scale) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const WT* wr = w + (size_t)row * cols;
  uint32_t* pr = reinterpret_cast<uint32_t*>(packed + (size_t)row * (cols >> 1));

  float srow = 0.f;
  if (!group) {
    float amax = 0.f;
    for (int c = lane; c < cols; c += 32) amax = fmaxf(amax, fabsf(to_f32<WT>(wr[c])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    srow = __fdiv_rn(amax, 7.0f);
    if (lane == 0) scale[row] = from_f32<ST>(srow);
  }
  for (int c0 = 0; c0 < cols; c0 += 128) {
    const int cb = c0 + lane * 4;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = cb + i < cols ? to_f32<WT>(wr[cb + i]) : 0.f;
    float s = srow;
    if (group) {
      float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      s = __fdiv_rn(amax, 7.0f);
      if (lane == 0) scale[(size_t)row * (cols / group) + c0 / group] = from_f32<ST>(s);
    }
    uint32_t part = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int q = 0;
      if (s != 0.f) {
        const float r = rintf(__fdiv_rn(v[i], s));
        q = (int)fminf(fmaxf(r, -8.f), 7.f);
      }
      const int c = (lane & 1) * 4 + i;
      part |= (uint32_t)((q + 8) & 0xF) << column_shift(packing, c);
    }
    part |= __shfl_xor_sync(0xffffffffu, part, 1);
    if ((lane & 1) == 0 && cb < cols) pr[cb >> 3] = part;
  }
}

int launch_quantize_pack(const void* w, int w_dtype, int rows, int cols, int group, int packing,
                         uint8_t* packed, void* scale, int scale_dtype, cudaStream_t stream) {
  const int grid = (rows + 7) / 8;
  const bool wf32 = w_dtype == W4A16_DTYPE_F32;
  const bool sf32 = scale_dtype == W4A16_DTYPE_F32;
  if (wf32 && sf32)
    k_quantize_pack<float, float><<<grid, 256, 0, stream>>>(
        static_cast<const float*>(w), rows, cols, group, packing, packed, static_cast<float*>(scale));
  else if (wf32)
    k_quantize_pack<float, __half><<<grid, 256, 0, stream>>>(
        static_cast<const float*>(w), rows, cols, group, packing, packed, static_cast<__half*>(scale));
  else if (sf32)
    k_quantize_pack<__half, float><<<grid, 256, 0, stream>>>(
        static_cast<const __half*>(w), rows, cols, group, packing, packed, static_cast<float*>(scale));
  else
    k_quantize_pack<__half, __half><<<grid, 256, 0, stream>>>(
        static_cast<const __half*>(w), rows, cols, group, packing, packed,
        static_cast<__half*>(scale));
  return check_launch("k_quantize_pack");
}

}  // namespace w4a16
