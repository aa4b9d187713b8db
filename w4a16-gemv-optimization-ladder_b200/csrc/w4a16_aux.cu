// Companion kernels of the W4A16 GEMV path (sm_100a):
//   k_h2f32           lossy variant: fp16 products summed in fp16 per packed word
//                     (reference k_h2f32, kernels/w4a16_kernels.cu:161-171)
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

// One warp per row.  Each packed word's eight products are formed and summed in
// fp16 (one mul + three fma on f16x2), then added to an fp32 accumulator.
__global__ void __launch_bounds__(256)
    k_h2f32(const uint8_t* __restrict__ packed, const float* __restrict__ scale,
            const __half* __restrict__ vec, float* __restrict__ out, int rows, int cols) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint32_t* wr = reinterpret_cast<const uint32_t*>(packed + (size_t)row * (cols >> 1));
  const int words = cols >> 3;
  float acc = 0.f;
  for (int w = lane; w < words; w += 32) {
    uint32_t o[4];
    decode_word(__ldg(wr + w), o);  // simple packing: pairs (1,5) (0,4) (3,7) (2,6)
    const uint4 xv = simple_order(ldg128(vec + (size_t)w * 8));
    uint32_t s = mul_f16x2(o[0], xv.x);
    s = fma_f16x2(o[1], xv.y, s);
    s = fma_f16x2(o[2], xv.z, s);
    s = fma_f16x2(o[3], xv.w, s);
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&s));
    acc += f.x + f.y;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) out[row] = acc * __ldg(scale + row);
}

int launch_h2f32(const uint8_t* packed, const float* scale, const void* vec, float* out, int rows,
                 int cols, cudaStream_t stream) {
  const int grid = (rows + 7) / 8;
  k_h2f32<<<grid, 256, 0, stream>>>(packed, scale, static_cast<const __half*>(vec), out, rows,
                                     cols);
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
