/*
 * TEST INFRASTRUCTURE ONLY — C restatement of the reference's W4A16 CPU algorithm.
 *
 * The same quantise / pack / dequant-then-matmul steps as oracle/w4a16_oracle.py
 * (which is pinned to the reference's golden vectors), in C with a pthread pool over
 * rows so that it finishes full-size shapes in seconds.  Used by tests/ to check the CUDA kernels at
 * the large configurations and by bench.py's CPU-baseline leg as the timed port of
 * the reference's torch CPU path.  The library itself never links or calls it.
 *
 * Reference steps restated (src/w4a16/kernels.py of
 * emirabayer/w4a16-gemv-optimization-ladder):
 *   quantize_int4_symmetric  :47-50   scale = max|w|/7, q = clamp(rint(w/scale),-8,7)
 *   quantize_int4_group      :52-60   the same per 128-column group
 *   pack_int4                :64-70   byte c = (q[2c]+8)<<4 | (q[2c+1]+8)
 *   pack_int4_interleaved    :73-91   nibble slot i of a u32 <- column {0,2,4,6,1,3,5,7}[i]
 *   dequant_ref(_group)      :94-101  y = (fp32(q) * scale) @ fp32(x)
 */
#include <math.h>
#include <pthread.h>
#include <unistd.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static const int kInterleave[8] = {0, 2, 4, 6, 1, 3, 5, 7};

static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  const uint32_t man = h & 0x3FFu;
  float v;
  if (exp == 0) {
    v = ldexpf((float)man, -24); /* zero or subnormal: man * 2^-24 */
    return sign ? -v : v;
  }
  uint32_t f = exp == 31 ? (sign | 0x7F800000u | (man << 13))
                         : (sign | ((exp + 112u) << 23) | (man << 13));
  memcpy(&v, &f, 4);
  return v;
}

/* Codes of one packed row, in column order. */
static void unpack_row(const uint8_t* row, int interleaved, int K, int8_t* q) {
  if (!interleaved) {
    for (int c = 0; c < K / 2; ++c) {
      q[2 * c] = (int8_t)((row[c] >> 4) - 8);
      q[2 * c + 1] = (int8_t)((row[c] & 0xF) - 8);
    }
    return;
  }
  for (int w = 0; w < K / 8; ++w) {
    const uint32_t word = (uint32_t)row[4 * w] | ((uint32_t)row[4 * w + 1] << 8) |
                          ((uint32_t)row[4 * w + 2] << 16) | ((uint32_t)row[4 * w + 3] << 24);
    for (int slot = 0; slot < 8; ++slot)
      q[8 * w + kInterleave[slot]] = (int8_t)(((word >> (4 * slot)) & 0xFu) - 8);
  }
}

/* Run body(lo, hi, ctx) over [0, n) split into `threads` contiguous ranges. */
typedef void (*range_fn)(int lo, int hi, void* ctx);
struct range_job {
  range_fn fn;
  void* ctx;
  int lo, hi;
};
static void* range_thread(void* arg) {
  struct range_job* j = (struct range_job*)arg;
  j->fn(j->lo, j->hi, j->ctx);
  return NULL;
}
int oracle_max_threads(void) {
  const long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}
static void parallel_rows(int n, int threads, range_fn fn, void* ctx) {
  if (threads <= 0) threads = oracle_max_threads();
  if (threads > n) threads = n > 0 ? n : 1;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  struct range_job job[256];
  for (int t = 0; t < threads; ++t) {
    job[t].fn = fn;
    job[t].ctx = ctx;
    job[t].lo = (int)((long long)n * t / threads);
    job[t].hi = (int)((long long)n * (t + 1) / threads);
  }
  for (int t = 1; t < threads; ++t) pthread_create(&tid[t], NULL, range_thread, &job[t]);
  range_thread(&job[0]);
  for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
}

struct gemv_ctx {
  const uint8_t* packed;
  int interleaved;
  const float* scale;
  int group;
  const float* xf;
  int M, N, K;
  float* y;
  int f64;
  int err;
};

static void gemv_rows(int lo, int hi, void* arg) {
  struct gemv_ctx* c = (struct gemv_ctx*)arg;
  const int K = c->K;
  int8_t* q = (int8_t*)malloc((size_t)K);
  float* wrow = (float*)malloc(sizeof(float) * (size_t)K);
  if (!q || !wrow) {
    c->err = -2;
    free(q);
    free(wrow);
    return;
  }
  for (int r = lo; r < hi; ++r) {
    unpack_row(c->packed + (size_t)r * (K / 2), c->interleaved, K, q);
    for (int k = 0; k < K; ++k) {
      const float s = c->group ? c->scale[(size_t)r * (K / c->group) + k / c->group] : c->scale[r];
      wrow[k] = (float)q[k] * s;
    }
    for (int m = 0; m < c->M; ++m) {
      const float* xm = c->xf + (size_t)m * K;
      if (c->f64) {
        double acc = 0.0;
        for (int k = 0; k < K; ++k) acc += (double)wrow[k] * (double)xm[k];
        c->y[(size_t)m * c->N + r] = (float)acc;
      } else {
        float part[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int k = 0; k < K; k += 8)
          for (int u = 0; u < 8; ++u) part[u] += wrow[k + u] * xm[k + u];
        float acc = 0.f;
        for (int u = 0; u < 8; ++u) acc += part[u];
        c->y[(size_t)m * c->N + r] = acc;
      }
    }
  }
  free(q);
  free(wrow);
}

/*
 * y[m][r] = sum_k fp32(q[r][k]) * scale(r,k) * fp32(x[m][k]).
 * The dequantised weight is rounded to fp32 as in the reference (q.float()*scale);
 * the dot product is summed in double (accumulate_f64 != 0, the checker) or in fp32
 * with 8 interleaved partial sums (the timed baseline, like a BLAS sgemv).
 * threads <= 0 uses one thread per online CPU.
 */
int oracle_gemv(const uint8_t* packed, int interleaved, const float* scale, int group,
                const uint16_t* x, int M, int N, int K, float* y, int accumulate_f64,
                int threads) {
  if (K % 8 || (group && K % group)) return -1;
  float* xf = (float*)malloc(sizeof(float) * (size_t)M * K);
  if (!xf) return -2;
  for (size_t i = 0; i < (size_t)M * K; ++i) xf[i] = half_to_float(x[i]);
  struct gemv_ctx c = {packed, interleaved, scale, group, xf, M, N, K, y, accumulate_f64, 0};
  parallel_rows(N, threads, gemv_rows, &c);
  free(xf);
  return c.err;
}

struct qp_ctx {
  const float* w;
  int cols, group, interleaved;
  uint8_t* packed;
  float* scale;
};

static void quantize_rows(int lo, int hi, void* arg) {
  struct qp_ctx* c = (struct qp_ctx*)arg;
  const int cols = c->cols, group = c->group;
  int8_t* q = (int8_t*)malloc((size_t)cols);
  for (int r = lo; r < hi; ++r) {
    const float* wr = c->w + (size_t)r * cols;
    const int span = group ? group : cols;
    for (int c0 = 0; c0 < cols; c0 += span) {
      float amax = 0.f;
      for (int k = c0; k < c0 + span; ++k) amax = fmaxf(amax, fabsf(wr[k]));
      const float s = amax / 7.0f;
      if (group)
        c->scale[(size_t)r * (cols / group) + c0 / group] = s;
      else
        c->scale[r] = s;
      for (int k = c0; k < c0 + span; ++k) {
        float v = s == 0.f ? 0.f : rintf(wr[k] / s);
        v = v < -8.f ? -8.f : (v > 7.f ? 7.f : v);
        q[k] = (int8_t)v;
      }
    }
    uint8_t* out = c->packed + (size_t)r * (cols / 2);
    if (!c->interleaved) {
      for (int k = 0; k < cols / 2; ++k)
        out[k] = (uint8_t)((((q[2 * k] + 8) & 0xF) << 4) | ((q[2 * k + 1] + 8) & 0xF));
    } else {
      for (int wi = 0; wi < cols / 8; ++wi) {
        uint32_t word = 0;
        for (int slot = 0; slot < 8; ++slot)
          word |= (uint32_t)((q[8 * wi + kInterleave[slot]] + 8) & 0xF) << (4 * slot);
        for (int b = 0; b < 4; ++b) out[4 * wi + b] = (uint8_t)(word >> (8 * b));
      }
    }
  }
  free(q);
}

/* Quantise fp32 w [rows][cols] and pack (scale fp32 [rows] or [rows][cols/group]). */
int oracle_quantize_pack(const float* w, int rows, int cols, int group, int interleaved,
                         uint8_t* packed, float* scale, int threads) {
  if (cols % 8 || (group && cols % group)) return -1;
  struct qp_ctx c = {w, cols, group, interleaved, packed, scale};
  parallel_rows(rows, threads, quantize_rows, &c);
  return 0;
}
