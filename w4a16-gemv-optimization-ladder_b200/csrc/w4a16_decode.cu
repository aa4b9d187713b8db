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

#include <atomic>

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

// Thread-block cluster helpers (the CL variant of k_decode_attention: one cluster per kv head).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// A float of CTA `rank`'s shared memory at the offset of `local` in this CTA's.
__device__ __forceinline__ float ld_cluster_f32(const float* local, unsigned rank) {
  uint32_t a = (uint32_t)__cvta_generic_to_shared(local), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}

// CL: the kv head's splits form one thread-block cluster; each CTA leaves its partial
// softmaxes in its own shared memory and split 0 combines them through distributed shared
// memory between two cluster barriers (no global round trips, fence or counter).
template <int MAXT, bool CL>
__global__ void __launch_bounds__(MAXT) k_decode_attention(const __half* qkv, const float* __restrict__ cos_t,
                                   const float* __restrict__ sin_t, const long long* __restrict__ pos_p,
                                   __half* k_cache, __half* v_cache, __half* __restrict__ out,
                                   float* __restrict__ scratch, int heads, int kv_heads, int max_len,
                                   int splits, float scale) {
  const int kvh = blockIdx.x / splits;
  const int split = blockIdx.x % splits;
  const int group = heads / kv_heads;
  const int warp = threadIdx.x >> 5;  // query head within the group
  const int lane = threadIdx.x & 31;
  const int head = kvh * group + warp;
  const long long pos_ll = pos_p[0];  // set before the step, not by the previous kernel
  const bool bad_pos = pos_ll < 0 || pos_ll >= max_len;
  const int pos = bad_pos ? 0 : (int)pos_ll;
  const int span = (max_len + splits - 1) / splits;
  const int j0 = split * span;
  const int j1 = min(min(j0 + span, max_len), pos + 1);
  __half* kc = k_cache + (size_t)kvh * max_len * kHeadDim;  // this kv head's rows
  __half* vc = v_cache + (size_t)kvh * max_len * kHeadDim;

  // Rows below pos were written by earlier steps, which have completed: when this CTA's
  // positions fit one block of 32, fetch its key row (one per lane) and the block's value
  // rows (dims 2 lane, 2 lane + 1) before waiting for the previous kernel.
  const bool one_block = span <= 32 && !bad_pos;
  const int j = j0 + lane;
  const int nvalid = max(0, j1 - j0);
  uint4 kreg[8];
  __half2 vreg[32];
  if (one_block) {
    if (j < j1 && j != pos) {
      const uint4* kr = reinterpret_cast<const uint4*>(kc + (size_t)j * kHeadDim);
#pragma unroll
      for (int e = 0; e < 8; ++e) kreg[e] = kr[e];
    }
    const __half2* vr = reinterpret_cast<const __half2*>(vc + (size_t)j0 * kHeadDim) + lane;
#pragma unroll
    for (int u = 0; u < 32; ++u)
      if (u < nvalid && j0 + u != pos) vreg[u] = vr[u * (kHeadDim / 2)];
  }

  // qkv (and, for span > 32, the new cache row) come from the kernels before this one
  grid_dependency_wait();
  grid_launch_dependents();
  if (bad_pos) {  // nothing is read or written: the heads read NaN
    if (split == 0) {
      const __half2 nan2 = __float2half2_rn(__int_as_float(0x7fc00000));
      reinterpret_cast<__half2*>(out + head * kHeadDim)[lane] = nan2;
    }
    return;
  }

  extern __shared__ float sm[];  // rotated, pre-scaled queries [group][64]; new key, value [64] each
  float* qs = sm;
  float* kn = sm + group * kHeadDim;
  float* vn = kn + kHeadDim;
  const float* cr = cos_t + (size_t)pos * kHeadDim;
  const float* sr = sin_t + (size_t)pos * kHeadDim;
  {  // rotate this warp's query head
    float a = __half2float(__ldcg(qkv + head * kHeadDim + lane));
    float b = __half2float(__ldcg(qkv + head * kHeadDim + lane + 32));
    rope_pair(a, b, cr, sr, lane);
    qs[warp * kHeadDim + lane] = a * scale;
    qs[warp * kHeadDim + lane + 32] = b * scale;
  }
  if (warp == 0 && pos >= j0 && pos < j0 + span) {
    // this split owns the new position: rotate the key, write key and value to the
    // cache and keep both (as fp16 values) for the loops below
    const int kb = heads * kHeadDim + kvh * kHeadDim;
    const int vb = (heads + kv_heads) * kHeadDim + kvh * kHeadDim;
    float a = __half2float(__ldcg(qkv + kb + lane));
    float b = __half2float(__ldcg(qkv + kb + lane + 32));
    rope_pair(a, b, cr, sr, lane);
    const __half ah = __float2half_rn(a), bh = __float2half_rn(b);
    const __half va = __ldcg(qkv + vb + lane), vb2 = __ldcg(qkv + vb + lane + 32);
    kc[(size_t)pos * kHeadDim + lane] = ah;
    kc[(size_t)pos * kHeadDim + lane + 32] = bh;
    vc[(size_t)pos * kHeadDim + lane] = va;
    vc[(size_t)pos * kHeadDim + lane + 32] = vb2;
    kn[lane] = __half2float(ah);
    kn[lane + 32] = __half2float(bh);
    vn[lane] = __half2float(va);
    vn[lane + 32] = __half2float(vb2);
  }
  __syncthreads();  // queries, the new row and the cache write are visible to the CTA

  // Partial softmax over [j0, j1): lane handles position jb + lane of each block of 32
  // for the scores, and dims (2 lane, 2 lane + 1) of the output.
  float m = -INFINITY, l = 0.f;
  float2 o = make_float2(0.f, 0.f);
  const float* q = qs + warp * kHeadDim;
  auto score = [&](const uint4* kv) {
    float d = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t w4[4] = {kv[e].x, kv[e].y, kv[e].z, kv[e].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
        d = fmaf(q[e * 8 + 2 * i], f.x, d);
        d = fmaf(q[e * 8 + 2 * i + 1], f.y, d);
      }
    }
    return d;
  };
  auto softmax_block = [&](float sc) {  // running max / sum update over a block; returns p_j
    const float mn = fmaxf(m, warp_max(sc));
    const float corr = m == -INFINITY ? 0.f : __expf(m - mn);
    const float pj = sc == -INFINITY ? 0.f : __expf(sc - mn);
    l = l * corr + warp_sum(pj);
    o.x *= corr;
    o.y *= corr;
    m = mn;
    return pj;
  };
  if (one_block) {
    float sc = -INFINITY;
    if (j < j1) {
      if (j == pos) {
        float d = 0.f;
#pragma unroll 8
        for (int e = 0; e < kHeadDim; ++e) d = fmaf(q[e], kn[e], d);
        sc = d;
      } else {
        sc = score(kreg);
      }
    }
    const float pj = softmax_block(sc);
#pragma unroll
    for (int u = 0; u < 32; ++u) {
      if (u < nvalid) {
        const float pu = __shfl_sync(0xffffffffu, pj, u);
        const float2 v = j0 + u == pos ? make_float2(vn[2 * lane], vn[2 * lane + 1]) : __half22float2(vreg[u]);
        o.x = fmaf(pu, v.x, o.x);
        o.y = fmaf(pu, v.y, o.y);
      }
    }
  } else {
    for (int jb = j0; jb < j1; jb += 32) {
      const int jj = jb + lane;
      float sc = -INFINITY;
      if (jj < j1) {
        const uint4* kr = reinterpret_cast<const uint4*>(kc + (size_t)jj * kHeadDim);
        uint4 kv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) kv[e] = kr[e];
        sc = score(kv);
      }
      const float pj = softmax_block(sc);
      const __half2* vr = reinterpret_cast<const __half2*>(vc + (size_t)jb * kHeadDim) + lane;
      const int nv = min(32, j1 - jb);
#pragma unroll
      for (int u = 0; u < 32; ++u)  // all value rows of the block in flight first
        if (u < nv) vreg[u] = vr[u * (kHeadDim / 2)];
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        if (u < nv) {
          const float pu = __shfl_sync(0xffffffffu, pj, u);
          const float2 v = __half22float2(vreg[u]);
          o.x = fmaf(pu, v.x, o.x);
          o.y = fmaf(pu, v.y, o.y);
        }
      }
    }
  }

  constexpr int kPart = kHeadDim + 2;
  if constexpr (CL) {
    // Every CTA of the cluster reaches both barriers (the only early return, a bad
    // position, is taken by all of them before either).
    float* cp = sm + (group + 2) * kHeadDim;  // [group][kPart]: this CTA's partials
    float* mine = cp + warp * kPart;
    if (lane == 0) {
      mine[0] = m;
      mine[1] = l;
    }
    mine[2 + 2 * lane] = o.x;
    mine[3 + 2 * lane] = o.y;
    cluster_sync_all();  // every split's partials are in place
    if (split == 0) {
      // lane s holds split s's max and weight; each lane gathers its two dims of every
      // split's output, summed in split order (splits <= 32)
      const float ms = lane < splits ? ld_cluster_f32(mine, (unsigned)lane) : -INFINITY;
      const float M = warp_max(ms);
      const float w = lane < splits && ms != -INFINITY ? __expf(ms - M) : 0.f;
      const float lw = lane < splits ? ld_cluster_f32(mine + 1, (unsigned)lane) * w : 0.f;
      float L = 0.f;
      float2 a = make_float2(0.f, 0.f);
      for (int u = 0; u < splits; ++u) {
        const float wu = __shfl_sync(0xffffffffu, w, u);
        L += __shfl_sync(0xffffffffu, lw, u);
        a.x = fmaf(ld_cluster_f32(mine + 2 + 2 * lane, (unsigned)u), wu, a.x);
        a.y = fmaf(ld_cluster_f32(mine + 3 + 2 * lane, (unsigned)u), wu, a.y);
      }
      reinterpret_cast<__half2*>(out + head * kHeadDim)[lane] = __floats2half2_rn(a.x / L, a.y / L);
    }
    cluster_sync_all();  // no CTA exits while split 0 reads its shared memory
    return;
  }
  // publish (m, l, o) for (head, split); the last split of this kv head combines
  float* part = scratch + ((size_t)head * splits + split) * kPart;
  if (lane == 0) {
    part[0] = m;
    part[1] = l;
  }
  reinterpret_cast<float2*>(part + 2)[lane] = o;
  __threadfence();
  __syncthreads();
  unsigned* counters = reinterpret_cast<unsigned*>(scratch + (size_t)heads * splits * kPart);
  __shared__ unsigned prev;
  if (threadIdx.x == 0) prev = atomicAdd(counters + kvh, 1u);
  __syncthreads();
  if (prev != (unsigned)(splits - 1)) return;
  __threadfence();
  // Combine the splits in split order, 32 at a time: lane s holds split s's max and
  // weight; each lane gathers its two dims of every split's output.
  const float* ph = scratch + (size_t)head * splits * kPart;
  float M = -INFINITY;
  for (int s = lane; s < splits; s += 32) M = fmaxf(M, __ldcg(ph + (size_t)s * kPart));
  M = warp_max(M);
  float L = 0.f;
  float2 a = make_float2(0.f, 0.f);
  for (int s0 = 0; s0 < splits; s0 += 32) {
    const int s = s0 + lane;
    float w = 0.f, lw = 0.f;
    if (s < splits) {
      const float ms = __ldcg(ph + (size_t)s * kPart);
      w = ms == -INFINITY ? 0.f : __expf(ms - M);
      lw = __ldcg(ph + (size_t)s * kPart + 1) * w;
    }
    float2 os[32];
#pragma unroll
    for (int u = 0; u < 32; ++u)
      if (s0 + u < splits) os[u] = __ldcg(reinterpret_cast<const float2*>(ph + (size_t)(s0 + u) * kPart + 2) + lane);
#pragma unroll
    for (int u = 0; u < 32; ++u) {
      const float wu = __shfl_sync(0xffffffffu, w, u);
      const float lu = __shfl_sync(0xffffffffu, lw, u);
      if (s0 + u < splits) {
        L += lu;
        a.x = fmaf(os[u].x, wu, a.x);
        a.y = fmaf(os[u].y, wu, a.y);
      }
    }
  }
  reinterpret_cast<__half2*>(out + head * kHeadDim)[lane] = __floats2half2_rn(a.x / L, a.y / L);
  __syncthreads();
  if (threadIdx.x == 0) counters[kvh] = 0u;
}

// One CTA per kv head for a cache of at most kCtaWarps * 32 positions and G query heads
// per kv head: warp w takes positions [32w, 32w + 32) for all G heads (one key row per
// lane), and the 16 warps' partial softmaxes are combined in shared memory, so nothing
// but the output leaves the CTA.  The key and value rows below pos are fetched before the
// dependency wait (earlier steps wrote them); warp G writes the new row at pos.
constexpr int kCtaWarps = 16;

template <int G>
__global__ void __launch_bounds__(kCtaWarps * 32)
    k_decode_attention_cta(const __half* qkv, const float* __restrict__ cos_t,
                           const float* __restrict__ sin_t, const long long* __restrict__ pos_p,
                           __half* k_cache, __half* v_cache, __half* __restrict__ out, int heads,
                           int kv_heads, int max_len, float scale) {
  static_assert(G >= 1 && G < kCtaWarps, "query heads per kv head");
  constexpr int kPart = kHeadDim + 2;
  const int kvh = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long pos_ll = pos_p[0];  // set before the step
  const bool bad_pos = pos_ll < 0 || pos_ll >= max_len;
  const int pos = bad_pos ? 0 : (int)pos_ll;
  const int jend = bad_pos ? 0 : pos + 1;  // positions [0, pos] take part
  const int j0 = warp * 32;
  const int j = j0 + lane;
  const int nvalid = max(0, min(32, jend - j0));
  __half* kc = k_cache + (size_t)kvh * max_len * kHeadDim;
  __half* vc = v_cache + (size_t)kvh * max_len * kHeadDim;

  uint4 kreg[8];
  __half2 vreg[32];
  if (j < jend && j != pos) {
    const uint4* kr = reinterpret_cast<const uint4*>(kc + (size_t)j * kHeadDim);
#pragma unroll
    for (int e = 0; e < 8; ++e) kreg[e] = kr[e];
  }
  {
    const __half2* vr = reinterpret_cast<const __half2*>(vc + (size_t)j0 * kHeadDim) + lane;
#pragma unroll
    for (int u = 0; u < 32; ++u)
      if (u < nvalid && j0 + u != pos) vreg[u] = vr[u * (kHeadDim / 2)];
  }

  grid_dependency_wait();
  grid_launch_dependents();
  if (bad_pos) {  // nothing is read or written: the heads read NaN
    if (warp < G) {
      const __half2 nan2 = __float2half2_rn(__int_as_float(0x7fc00000));
      reinterpret_cast<__half2*>(out + (kvh * G + warp) * kHeadDim)[lane] = nan2;
    }
    return;
  }

  extern __shared__ float sm[];  // q [G][64] (rotated, scaled) | k_new [64] | v_new [64] | parts [warps][G][66]
  float* qs = sm;
  float* kn = qs + G * kHeadDim;
  float* vn = kn + kHeadDim;
  float* parts = vn + kHeadDim;
  const float* cr = cos_t + (size_t)pos * kHeadDim;
  const float* sr = sin_t + (size_t)pos * kHeadDim;
  if (warp < G) {  // rotate query head kvh * G + warp
    const int head = kvh * G + warp;
    float a = __half2float(__ldcg(qkv + head * kHeadDim + lane));
    float b = __half2float(__ldcg(qkv + head * kHeadDim + lane + 32));
    rope_pair(a, b, cr, sr, lane);
    qs[warp * kHeadDim + lane] = a * scale;
    qs[warp * kHeadDim + lane + 32] = b * scale;
  } else if (warp == G) {  // the new key (rotated) and value, into the cache and smem
    const int kb = heads * kHeadDim + kvh * kHeadDim;
    const int vb = (heads + kv_heads) * kHeadDim + kvh * kHeadDim;
    float a = __half2float(__ldcg(qkv + kb + lane));
    float b = __half2float(__ldcg(qkv + kb + lane + 32));
    rope_pair(a, b, cr, sr, lane);
    const __half ah = __float2half_rn(a), bh = __float2half_rn(b);
    const __half va = __ldcg(qkv + vb + lane), vb2 = __ldcg(qkv + vb + lane + 32);
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

  // this warp's block for every query head of the group
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const float* q = qs + h * kHeadDim;
    float sc = -INFINITY;
    if (j < jend) {
      float d = 0.f;
      if (j == pos) {
#pragma unroll 8
        for (int e = 0; e < kHeadDim; ++e) d = fmaf(q[e], kn[e], d);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint32_t w4[4] = {kreg[e].x, kreg[e].y, kreg[e].z, kreg[e].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
            d = fmaf(q[e * 8 + 2 * i], f.x, d);
            d = fmaf(q[e * 8 + 2 * i + 1], f.y, d);
          }
        }
      }
      sc = d;
    }
    const float m = warp_max(sc);
    const float pj = sc == -INFINITY ? 0.f : __expf(sc - m);
    const float l = warp_sum(pj);
    float2 o = make_float2(0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 32; ++u) {
      if (u < nvalid) {
        const float pu = __shfl_sync(0xffffffffu, pj, u);
        const float2 v = j0 + u == pos ? make_float2(vn[2 * lane], vn[2 * lane + 1])
                                       : __half22float2(vreg[u]);
        o.x = fmaf(pu, v.x, o.x);
        o.y = fmaf(pu, v.y, o.y);
      }
    }
    float* part = parts + (warp * G + h) * kPart;
    if (lane == 0) {
      part[0] = m;  // -inf for a block past pos
      part[1] = l;
    }
    reinterpret_cast<float2*>(part + 2)[lane] = o;
  }
  __syncthreads();

  if (warp < G) {  // head kvh * G + warp: combine the blocks in warp order
    const int h = warp;
    const float mw = lane < kCtaWarps ? parts[(lane * G + h) * kPart] : -INFINITY;
    const float M = warp_max(mw);
    const float ww = mw == -INFINITY ? 0.f : __expf(mw - M);
    const float lw = lane < kCtaWarps ? parts[(lane * G + h) * kPart + 1] * ww : 0.f;
    float L = 0.f;
    float2 a = make_float2(0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kCtaWarps; ++w) {
      const float wu = __shfl_sync(0xffffffffu, ww, w);
      L += __shfl_sync(0xffffffffu, lw, w);
      const float2 ov = reinterpret_cast<const float2*>(parts + (w * G + h) * kPart + 2)[lane];
      a.x = fmaf(ov.x, wu, a.x);
      a.y = fmaf(ov.y, wu, a.y);
    }
    reinterpret_cast<__half2*>(out + (kvh * G + h) * kHeadDim)[lane] = __floats2half2_rn(a.x / L, a.y / L);
  }
}

}  // namespace

size_t decode_attention_scratch_bytes(int heads, int kv_heads, int splits) {
  return ((size_t)heads * splits * (kHeadDim + 2) + (size_t)kv_heads) * 4;
}

int launch_decode_attention(const void* qkv, const float* cos_t, const float* sin_t,
                            const long long* pos, void* k_cache, void* v_cache, void* out,
                            void* scratch, int heads, int kv_heads, int head_dim, int max_len,
                            int splits, bool pdl, cudaStream_t stream) {
  const int group = heads / kv_heads;
  if (splits == 1 && max_len <= kCtaWarps * 32 && (group == 1 || group == 2 || group == 4 || group == 8)) {
    // the whole cache of a kv head in one CTA: combine in shared memory
    const size_t csmem = ((size_t)(group + 2) * kHeadDim + (size_t)kCtaWarps * group * (kHeadDim + 2)) * 4;
    auto ck = group == 1 ? k_decode_attention_cta<1>
                         : group == 2 ? k_decode_attention_cta<2>
                                      : group == 4 ? k_decode_attention_cta<4> : k_decode_attention_cta<8>;
    cudaError_t e = launch_maybe_pdl(
        ck, dim3(kv_heads), dim3(kCtaWarps * 32), csmem, stream, pdl, static_cast<const __half*>(qkv),
        cos_t, sin_t, pos, static_cast<__half*>(k_cache), static_cast<__half*>(v_cache),
        static_cast<__half*>(out), heads, kv_heads, max_len, 1.0f / sqrtf((float)head_dim));
    (void)cudaGetLastError();
    if (e != cudaSuccess) {
      set_error("k_decode_attention_cta launch failed: %s", cudaGetErrorString(e));
      return W4A16_ERR_CUDA;
    }
    return W4A16_OK;
  }
  const size_t smem = (size_t)(group + 2) * kHeadDim * 4;
  // One thread-block cluster per kv head (2..16 splits, up to 8 query heads): the splits
  // combine through distributed shared memory.  Used when the device can co-schedule such a
  // cluster (checked once per device and cluster size), else the global-memory combine.
  if (group <= 8 && splits >= 2 && splits <= 16) {
    static std::atomic<uint64_t> tried[17], usable[17];
    int dev = 0;
    (void)cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    auto ck = k_decode_attention<256, true>;
    const size_t csm = smem + (size_t)group * (kHeadDim + 2) * 4;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kv_heads * splits);
    cfg.blockDim = dim3(32 * group);
    cfg.dynamicSmemBytes = csm;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    if (!(tried[splits].load(std::memory_order_acquire) & bit)) {
      bool ok = cudaFuncSetAttribute(ck, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
      int nclusters = 0;
      cfg.numAttrs = 1;
      ok = ok && cudaOccupancyMaxActiveClusters(&nclusters, ck, &cfg) == cudaSuccess && nclusters > 0;
      (void)cudaGetLastError();
      if (ok) usable[splits].fetch_or(bit, std::memory_order_acq_rel);
      tried[splits].fetch_or(bit, std::memory_order_acq_rel);
    }
    if (usable[splits].load(std::memory_order_acquire) & bit) {
      cfg.numAttrs = pdl ? 2 : 1;
      cudaError_t e = cudaLaunchKernelEx(&cfg, ck, static_cast<const __half*>(qkv), cos_t, sin_t, pos,
                                         static_cast<__half*>(k_cache), static_cast<__half*>(v_cache),
                                         static_cast<__half*>(out), static_cast<float*>(scratch), heads,
                                         kv_heads, max_len, splits, 1.0f / sqrtf((float)head_dim));
      (void)cudaGetLastError();
      if (e != cudaSuccess) {
        set_error("k_decode_attention (cluster) launch failed: %s", cudaGetErrorString(e));
        return W4A16_ERR_CUDA;
      }
      return W4A16_OK;
    }
  }
  // up to 8 query heads per kv head (256 threads) the prefetch keeps its registers;
  // larger groups run with the register cap of 1024-thread blocks
  auto kernel = group <= 8 ? k_decode_attention<256, false> : k_decode_attention<1024, false>;
  cudaError_t e = launch_maybe_pdl(
      kernel, dim3(kv_heads * splits), dim3(32 * group), smem, stream, pdl,
      static_cast<const __half*>(qkv), cos_t, sin_t, pos, static_cast<__half*>(k_cache),
      static_cast<__half*>(v_cache), static_cast<__half*>(out), static_cast<float*>(scratch), heads,
      kv_heads, max_len, splits, 1.0f / sqrtf((float)head_dim));
  (void)cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("k_decode_attention launch failed: %s", cudaGetErrorString(e));
    return W4A16_ERR_CUDA;
  }
  return W4A16_OK;
}

}  // namespace w4a16
