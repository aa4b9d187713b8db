// Decode-step attention for Llama-style models (one token, batch 1), fused with the
// rotary embedding and the KV-cache write.  Not on the reference's path (it used the
// Hugging Face attention around its GEMVs); this is the part of a decode step that sits
// between the QKV GEMV and the output-projection GEMV.
//
// Grid: kv_heads x splits CTAs of 32 * (heads / kv_heads) threads, one warp per query
// head of the group.  CTA (kvh, s) rotates the query heads of its group and its key
// head, writes the new key and value into the cache at `pos` if position `pos` is in
// its range, and computes a partial softmax over positions [s*span, (s+1)*span) ∩
// [0, pos]: running max m, sum l and the unnormalised output o (fp32).  The last CTA
// of each head (an atomic counter in `scratch`, no waiting) combines the partials in
// split order and writes the fp16 output; it leaves the counter at zero.  A position
// outside [0, max_len) touches neither cache and makes every output NaN.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "w4a16_device.cuh"
#include "w4a16_internal.h"

namespace w4a16 {

namespace {

constexpr int kHeadDim = 64;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Rotate-half rotary embedding of one 64-dim head held as lane pair (lane, lane+32):
// lane i < 32 owns dims i and i + 32.
__device__ __forceinline__ void rope_pair(float& a, float& b, const float* cos_row,
                                          const float* sin_row, int lane) {
  const float c0 = cos_row[lane], s0 = sin_row[lane];
  const float c1 = cos_row[lane + 32], s1 = sin_row[lane + 32];
  const float ra = a * c0 - b * s0;
  const float rb = b * c1 + a * s1;
  a = ra;
  b = rb;
}

__global__ void k_decode_attention(const __half* __restrict__ qkv, const float* __restrict__ cos_t,
                                   const float* __restrict__ sin_t, const long long* __restrict__ pos_p,
                                   __half* __restrict__ k_cache, __half* __restrict__ v_cache,
                                   __half* __restrict__ out, float* __restrict__ scratch, int heads,
                                   int kv_heads, int max_len, int splits, float scale) {
  const int kvh = blockIdx.x / splits;
  const int split = blockIdx.x % splits;
  const int group = heads / kv_heads;
  const int warp = threadIdx.x >> 5;  // query head within the group
  const int lane = threadIdx.x & 31;
  const int head = kvh * group + warp;
  const long long pos_ll = pos_p[0];
  if (pos_ll < 0 || pos_ll >= max_len) {  // nothing is read or written: the heads read NaN
    if (split == 0) {
      out[head * kHeadDim + lane] = __float2half_rn(__int_as_float(0x7fc00000));
      out[head * kHeadDim + lane + 32] = __float2half_rn(__int_as_float(0x7fc00000));
    }
    return;
  }
  const int pos = (int)pos_ll;
  const int span = (max_len + splits - 1) / splits;
  const int j0 = split * span;
  const int j1 = min(min(j0 + span, max_len), pos + 1);

  extern __shared__ float sm[];  // q [group][64], k_new [64], v_new [64]
  float* qs = sm;
  float* kn = sm + group * kHeadDim;
  float* vn = kn + kHeadDim;

  const float* cr = cos_t + (size_t)pos * kHeadDim;
  const float* sr = sin_t + (size_t)pos * kHeadDim;
  {  // rotate this warp's query head
    float a = __half2float(qkv[head * kHeadDim + lane]);
    float b = __half2float(qkv[head * kHeadDim + lane + 32]);
    rope_pair(a, b, cr, sr, lane);
    qs[warp * kHeadDim + lane] = a * scale;
    qs[warp * kHeadDim + lane + 32] = b * scale;
  }
  if (warp == 0) {  // the new key (rotated) and value of this kv head
    const int kb = heads * kHeadDim + kvh * kHeadDim;
    const int vb = (heads + kv_heads) * kHeadDim + kvh * kHeadDim;
    float a = __half2float(qkv[kb + lane]);
    float b = __half2float(qkv[kb + lane + 32]);
    rope_pair(a, b, cr, sr, lane);
    const __half ah = __float2half_rn(a), bh = __float2half_rn(b);  // as the cache holds it
    kn[lane] = __half2float(ah);
    kn[lane + 32] = __half2float(bh);
    vn[lane] = __half2float(qkv[vb + lane]);
    vn[lane + 32] = __half2float(qkv[vb + lane + 32]);
    if (pos >= j0 && pos < j0 + span) {  // this split owns the new position
      __half* kd = k_cache + ((size_t)kvh * max_len + pos) * kHeadDim;
      __half* vd = v_cache + ((size_t)kvh * max_len + pos) * kHeadDim;
      kd[lane] = ah;
      kd[lane + 32] = bh;
      vd[lane] = qkv[vb + lane];
      vd[lane + 32] = qkv[vb + lane + 32];
    }
  }
  __syncthreads();

  // partial softmax over [j0, j1): lane handles positions j0 + lane, j0 + lane + 32, ...
  float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f;  // o: dims lane, lane + 32
  const float* q = qs + warp * kHeadDim;
  for (int jb = j0; jb < j1; jb += 32) {
    const int j = jb + lane;
    float sc = -INFINITY;
    if (j < j1) {
      float d = 0.f;
      if (j == pos) {
#pragma unroll 8
        for (int e = 0; e < kHeadDim; ++e) d = fmaf(q[e], kn[e], d);
      } else {
        const __half* kr = k_cache + ((size_t)kvh * max_len + j) * kHeadDim;
#pragma unroll
        for (int e = 0; e < kHeadDim; e += 8) {
          const uint4 kv = ldg128(kr + e);
          const uint32_t w4[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
            d = fmaf(q[e + 2 * i], f.x, d);
            d = fmaf(q[e + 2 * i + 1], f.y, d);
          }
        }
      }
      sc = d;
    }
    const float mb = warp_max(sc);
    const float mn = fmaxf(m, mb);
    const float corr = m == -INFINITY ? 0.f : __expf(m - mn);
    const float pj = sc == -INFINITY ? 0.f : __expf(sc - mn);
    l = l * corr + warp_sum(pj);
    o0 *= corr;
    o1 *= corr;
    const int nvalid = min(32, j1 - jb);
    for (int u = 0; u < nvalid; ++u) {  // o += p_u * v_u
      const float pu = __shfl_sync(0xffffffffu, pj, u);
      const int ju = jb + u;
      float v0, v1;
      if (ju == pos) {
        v0 = vn[lane];
        v1 = vn[lane + 32];
      } else {
        const __half* vr = v_cache + ((size_t)kvh * max_len + ju) * kHeadDim;
        v0 = __half2float(vr[lane]);
        v1 = __half2float(vr[lane + 32]);
      }
      o0 = fmaf(pu, v0, o0);
      o1 = fmaf(pu, v1, o1);
    }
    m = mn;
  }

  // publish (m, l, o) for (head, split); the last split of this kv head combines
  float* part = scratch + ((size_t)head * splits + split) * (kHeadDim + 2);
  if (lane == 0) {
    part[0] = m;
    part[1] = l;
  }
  part[2 + lane] = o0;
  part[2 + lane + 32] = o1;
  __threadfence();
  __syncthreads();
  unsigned* counters = reinterpret_cast<unsigned*>(scratch + (size_t)heads * splits * (kHeadDim + 2));
  __shared__ unsigned prev;
  if (threadIdx.x == 0) prev = atomicAdd(counters + kvh, 1u);
  __syncthreads();
  if (prev != (unsigned)(splits - 1)) return;
  __threadfence();
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s)
    M = fmaxf(M, __ldcg(scratch + ((size_t)head * splits + s) * (kHeadDim + 2)));
  float L = 0.f, a0 = 0.f, a1 = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float* ps = scratch + ((size_t)head * splits + s) * (kHeadDim + 2);
    const float ms = __ldcg(ps);
    if (ms == -INFINITY) continue;
    const float w = __expf(ms - M);
    L = fmaf(__ldcg(ps + 1), w, L);
    a0 = fmaf(__ldcg(ps + 2 + lane), w, a0);
    a1 = fmaf(__ldcg(ps + 2 + lane + 32), w, a1);
  }
  out[head * kHeadDim + lane] = __float2half_rn(a0 / L);
  out[head * kHeadDim + lane + 32] = __float2half_rn(a1 / L);
  __syncthreads();
  if (threadIdx.x == 0) counters[kvh] = 0u;
}

}  // namespace

size_t decode_attention_scratch_bytes(int heads, int kv_heads, int splits) {
  return ((size_t)heads * splits * (kHeadDim + 2) + (size_t)kv_heads) * 4;
}

int launch_decode_attention(const void* qkv, const float* cos_t, const float* sin_t,
                            const long long* pos, void* k_cache, void* v_cache, void* out,
                            void* scratch, int heads, int kv_heads, int head_dim, int max_len,
                            int splits, cudaStream_t stream) {
  const int group = heads / kv_heads;
  const size_t smem = (size_t)(group + 2) * kHeadDim * 4;
  k_decode_attention<<<kv_heads * splits, 32 * group, smem, stream>>>(
      static_cast<const __half*>(qkv), cos_t, sin_t, pos, static_cast<__half*>(k_cache),
      static_cast<__half*>(v_cache), static_cast<__half*>(out), static_cast<float*>(scratch), heads,
      kv_heads, max_len, splits, rsqrtf((float)head_dim));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("k_decode_attention launch failed: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  return W4A16_OK;
}

}  // namespace w4a16
