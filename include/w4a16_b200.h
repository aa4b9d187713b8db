/*
 * w4a16_b200.h — C ABI of the B200 (sm_100a) W4A16 GEMV library.
 *
 * Int4-weight x fp16-activation matrix-vector products with symmetric per-row or
 * group-128 scales.  Every entry point takes plain device pointers, sizes and a
 * CUDA stream, launches asynchronously on that stream, never synchronises (except
 * w4a16_read_device_error), never throws, and returns a status code (enum
 * w4a16_status).  Buffers are owned by the caller.
 *
 * The reference exposes its kernels as a pybind11 module compiled from
 * kernels/w4a16_kernels.cu (bindings at kernels/w4a16_kernels.cu:189-195, host
 * wrappers at :183-187, Python surface at src/w4a16/kernels.py:33-43).  Each
 * "*_cuda" function below replaces the binding of the same name; where the
 * reference allocated the output (kernels/w4a16_kernels.cu:183), the caller passes
 * it here.
 *
 * Layouts (row-major, contiguous):
 *   packed  uint8  [rows][cols/2]   int4 codes + 8, interleaved or simple packing
 *                                   (src/w4a16/kernels.py:64-91)
 *   scale   fp32 or fp16 [rows] (per-row) or [rows][cols/128] (group-128)
 *   vec / x fp16   [cols] or [batch][cols]
 *   out     fp32 (or fp16 via w4a16_gemv) [rows] or [batch][rows]
 * Requirements: cols % 8 == 0 (cols % 128 == 0 for group-128), vec/x 16-byte
 * aligned, packed 4-byte aligned, scale/out aligned to their element size.
 * rows == 0 or batch == 0 is a no-op that returns W4A16_OK.
 */
#ifndef W4A16_B200_H
#define W4A16_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st* w4a16_stream_t;

enum w4a16_status {
  W4A16_OK = 0,
  W4A16_ERR_NULL = -1,      /* a required pointer is NULL */
  W4A16_ERR_SHAPE = -2,     /* rows/cols/batch out of range, or cols not a multiple of 8 (128) */
  W4A16_ERR_ALIGN = -3,     /* a pointer is not aligned as required */
  W4A16_ERR_DTYPE = -4,     /* unknown dtype, packing or group code */
  W4A16_ERR_WORKSPACE = -5, /* workspace smaller than w4a16_gemv_workspace_bytes() for a split */
  W4A16_ERR_CUDA = -6,      /* a CUDA runtime call or kernel launch failed */
  W4A16_ERR_KERNEL = -7     /* a kernel gave up on a bounded wait (w4a16_read_device_error) */
};

enum w4a16_dtype { W4A16_DTYPE_F32 = 0, W4A16_DTYPE_F16 = 1 };
enum w4a16_packing { W4A16_PACK_INTERLEAVED = 0, W4A16_PACK_SIMPLE = 1 };
enum w4a16_prologue { W4A16_PROLOGUE_NONE = 0, W4A16_PROLOGUE_RMSNORM = 1, W4A16_PROLOGUE_SWIGLU = 2 };

/* Launch flags of the decode-step entries (w4a16_gemv_fused, w4a16_decode_attention).
 * W4A16_LAUNCH_PDL: programmatic dependent launch.  The kernel may start while the
 * previous kernel in the stream is still running: it loads its weights, then waits for
 * that kernel to finish before reading anything the kernel wrote, and lets the next
 * kernel start in turn.  Use it between these entries (a normal launch before or after
 * is unaffected); two consecutive calls must not share a workspace or scratch buffer. */
enum w4a16_launch_flags { W4A16_LAUNCH_PDL = 1, W4A16_LAUNCH_SWIGLU_OUT = 2 };

/* ---------------------------------------------------------------------------
 * Reference-mirroring entry points: out[r] = sum_k q[r][k] * scale * vec[k], fp32.
 * ------------------------------------------------------------------------- */

/* Replaces marlin_cuda (kernels/w4a16_kernels.cu:185,192 -> k_marlin :100-114;
 * Python w4a16_gemv, src/w4a16/kernels.py:40). Interleaved packing, per-row scale. */
int w4a16_marlin_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                      int rows, int cols, w4a16_stream_t stream);

/* Replaces marlin_g128_cuda (kernels/w4a16_kernels.cu:185,192 -> k_marlin_g128 :121-138;
 * Python w4a16_gemv_g128, src/w4a16/kernels.py:41). Interleaved packing, scale
 * fp32 [rows][cols/128]. */
int w4a16_marlin_g128_cuda(const uint8_t* packed, const float* scale, const void* vec,
                           float* out, int rows, int cols, w4a16_stream_t stream);

/* Replace the simple-packing ladder bindings byte_cuda, u32_cuda, u32_v4_cuda,
 * champ_cuda and uint4_cuda (kernels/w4a16_kernels.cu:184-185,190-193 -> k_byte
 * :50-56, k_u32 :59-69, k_u32_v4 :72-82, k_champ :85-96, k_uint4 :147-157; Python
 * matvec_*, src/w4a16/kernels.py:33-37).  All five run the same sm_100a kernel on
 * the simple packing, per-row fp32 scale, fp32 accumulation. */
int w4a16_byte_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                    int rows, int cols, w4a16_stream_t stream);
int w4a16_u32_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                   int rows, int cols, w4a16_stream_t stream);
int w4a16_u32_v4_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                      int rows, int cols, w4a16_stream_t stream);
int w4a16_champ_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                     int rows, int cols, w4a16_stream_t stream);
int w4a16_uint4_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                     int rows, int cols, w4a16_stream_t stream);

/* Replaces h2f32_cuda (kernels/w4a16_kernels.cu:185,194 -> k_h2f32 :161-171; Python
 * matvec_h2f32, src/w4a16/kernels.py:38).  Deliberately lossy: the eight products of
 * each packed word are multiplied and summed in fp16 before the fp32 accumulation.
 * Simple packing, per-row fp32 scale. */
int w4a16_h2f32_cuda(const uint8_t* packed, const float* scale, const void* vec, float* out,
                     int rows, int cols, w4a16_stream_t stream);

/* Replaces fp16_cuda (kernels/w4a16_kernels.cu:187,194 -> k_fp16 :174-180; Python
 * matvec_fp16, src/w4a16/kernels.py:43).  Dense fp16 mat [rows][cols] times fp16 vec,
 * fp32 accumulation and output.  cols % 8 == 0, mat and vec 16-byte aligned. */
int w4a16_fp16_cuda(const void* mat, const void* vec, float* out, int rows, int cols,
                    w4a16_stream_t stream);

/* ---------------------------------------------------------------------------
 * General entry point (superset of the bindings above).
 * ------------------------------------------------------------------------- */

/* out[b][r] = sum_k q[r][k] * scale(r, k) * x[b][k]  (+ bias[r]), b < batch.
 * The kernels behind w4a16_marlin_cuda / w4a16_marlin_g128_cuda (and, with the
 * simple packing, the ladder bindings) generalised to: fp16 or fp32 scales, a batch
 * of up to any number of activation rows (tensor-core path handles 16 per pass), an
 * fp16 or fp32 output, an optional fp32 bias (the epilogue W4A16Linear.forward
 * applies at src/w4a16/kernels.py:122-124), and split-K for short-row layers.
 *   group      0 (one scale per row) or 128 (one scale per 128 columns)
 *   workspace  NULL, or a zero-filled device buffer of workspace_bytes; when at
 *              least w4a16_gemv_workspace_bytes(batch, rows, cols) it lets every
 *              warp take an equal share of the work (tiles shared by two warps are
 *              reduced through it); without it each warp owns whole 16-row tiles.
 *              The kernels leave its counter block zeroed, so zero-filling once is
 *              enough (the partial sums are scratch).  Calls that share a workspace must be
 *              ordered on one stream.  Exception: after w4a16_read_device_error reports a
 *              non-zero code, a warp may have returned early and left counters behind:
 *              zero-fill again every workspace used since the previous read. */
int w4a16_gemv(const uint8_t* packed, int packing, const void* scale, int scale_dtype, int group,
               const void* x, int batch, int rows, int cols, void* out, int out_dtype,
               const float* bias, void* workspace, size_t workspace_bytes,
               w4a16_stream_t stream);

/* w4a16_gemv for one activation vector held in shared memory, the GEMV of a decode
 * step of a Llama-style model, with the activation optionally computed inside the
 * kernel.  The reference applies these operations as separate torch ops between its
 * GEMVs (the HF model around W4A16Linear, src/w4a16/kernels.py:113-124); here they are
 * the prologue of the GEMV that consumes them:
 *   W4A16_PROLOGUE_NONE     src = fp16 x [cols]
 *   W4A16_PROLOGUE_RMSNORM  src = fp32 h [cols], gamma = fp32 [cols]:
 *                           x = fp16(h * rsqrt(mean(h^2) + eps) * gamma)
 *   W4A16_PROLOGUE_SWIGLU   src = fp16 [2*cols] = gate | up:  x = fp16(silu(gate) * up)
 * One activation vector; interleaved packing; cols % 256 == 0 and small enough for the
 * vector to sit in shared memory beside the weight rings (cols <= 10752 with group-128
 * fp32 scales, <= 16640 with one scale per row).  out (fp32 or fp16 [rows]) may alias
 * bias (fp32): out = W x + bias is then an in-place residual add.  out must not overlap
 * src.  flags: W4A16_LAUNCH_PDL and, with the RMSNorm prologue only,
 * W4A16_LAUNCH_SWIGLU_OUT: the rows are gate / up pairs in blocks of 16 (rows 16b..16b+7
 * the gate rows and 16b+8..16b+15 the up rows of outputs 8b..8b+7), and out holds
 * rows / 2 values out[8b+i] = silu(y[16b+i]) * y[16b+8+i] of y = W x in fp32, rounded
 * once to out_dtype (a Llama MLP's gate|up projection with its activation applied in the
 * epilogue); rows % 16 == 0 and bias == NULL. */
int w4a16_gemv_fused(const uint8_t* packed, const void* scale, int scale_dtype, int group,
                     int prologue, const void* src, const float* gamma, float eps, int rows,
                     int cols, void* out, int out_dtype, const float* bias, void* workspace,
                     size_t workspace_bytes, unsigned flags, w4a16_stream_t stream);

/* Decode-step attention of a Llama-style layer for one token (batch 1), the kernel
 * that sits between the QKV and output GEMVs of a decode step.  The reference leaves
 * this to the Hugging Face model around its swapped Linears (benchmarks/end_to_end.py:
 * 24-42); here one launch does, at position p = *pos (device int64):
 *   q, k = rotary(qkv[q], qkv[k]) with rotate-half tables cos_t/sin_t (fp32 [max_len][64])
 *   k_cache[kvh][p] = fp16(k), v_cache[kvh][p] = qkv[v]          (fp16 [kv_heads][max_len][64])
 *   out[h] = softmax(q_h . k_cache[kvh(h)][0..p] / 8) @ v_cache[kvh(h)][0..p]   (fp16 [heads*64])
 * qkv = fp16 [(heads + 2*kv_heads) * 64] laid out q | k | v; head_dim must be 64 and
 * heads / kv_heads <= 32.  Positions are split over `splits` CTAs per kv head whose
 * fp32 partial softmaxes are combined: with 2..16 splits and <= 8 query heads per kv
 * head, by the first CTA of a thread-block cluster (one per kv head) through distributed
 * shared memory, when the device can co-schedule such a cluster; otherwise by the last CTA
 * to finish, through scratch and a per-kv-head counter.  scratch is a zero-filled device
 * buffer of w4a16_decode_attention_scratch_bytes(heads, kv_heads, splits) bytes that the
 * kernel leaves zeroed.  A position outside [0, max_len) writes nothing to the caches and
 * NaN to out.  Calls sharing a scratch buffer must be ordered on one stream.  flags: 0 or
 * W4A16_LAUNCH_PDL. */
int w4a16_decode_attention(const void* qkv, const float* cos_t, const float* sin_t,
                           const int64_t* pos, void* k_cache, void* v_cache, void* out,
                           void* scratch, size_t scratch_bytes, int heads, int kv_heads,
                           int head_dim, int max_len, int splits, unsigned flags,
                           w4a16_stream_t stream);

size_t w4a16_decode_attention_scratch_bytes(int heads, int kv_heads, int splits);

/* Tensor parallel with the all-gather fused into the GEMV (no counterpart in the
 * reference, which has one GPU; the unfused form is the local GEMV followed by
 * ncclAllGather).  Every rank owns one region of w4a16_tp_header_bytes() + the gathered
 * output's bytes, allocated by w4a16_tp_region_alloc on its GPU (zero-filled), and opens
 * the other ranks' regions from their IPC handles (w4a16_tp_region_open; handle size
 * w4a16_tp_ipc_handle_bytes()).  All ranks start from freshly allocated regions and make
 * the same sequence of calls on their streams. */
size_t w4a16_tp_header_bytes(void);
size_t w4a16_tp_ipc_handle_bytes(void);
int w4a16_tp_region_alloc(size_t out_bytes, void** region, void* ipc_handle);
int w4a16_tp_region_open(const void* ipc_handle, void** region);
int w4a16_tp_region_close(void* region, int owned);
/* The last fused step's timeline of a region's owner (a region allocated or opened in this
 * process; the owner's kernel writes it into its own region's header): four
 * %globaltimer stamps in ns — [0] this rank's start flags published, [1] every rank's start
 * flag seen (first warp of the first CTA), [2] this rank's rows stored and fenced (just before
 * its done flags), [3] every rank's done flag seen.  Synchronises `stream`. */
int w4a16_tp_region_timeline(const void* region, unsigned long long* stamps, w4a16_stream_t stream);

/* One step, one kernel: this rank's rows [row0, row0 + rows) of y = W x (interleaved
 * packing, one fp16 vector x [cols], out_dtype fp32 or fp16) are written by the GEMV's
 * epilogue straight into the gathered output of every rank (regions[k] +
 * w4a16_tp_header_bytes(), NVLink stores to the peers).  Each rank announces the step when
 * its kernel starts; a warp stores into other ranks' buffers only once every rank has
 * announced it (so no rank overwrites a buffer a peer is still reading from the previous
 * step); the kernel's last CTA publishes this rank's completion and waits for every rank's,
 * so when the call completes on the stream the gathered output is whole on this rank.
 * Waits are bounded (2 s by default, w4a16_tp_set_peer_wait_ns): a missing peer sets the
 * device error word (w4a16_read_device_error, code 2) and the step then writes this rank's
 * own rows only; the ranks' step numbers no longer agree after that, so close the regions
 * and allocate new ones before the next step.
 * regions: host array of nranks device pointers (own region at index rank), each returned by
 * w4a16_tp_region_alloc or w4a16_tp_region_open in this process; rows [row0, row0 + rows) must
 * fit the gathered output of every region (out_bytes given to w4a16_tp_region_alloc), else
 * W4A16_ERR_SHAPE with nothing launched.  Stream-ordered and graph-capturable: step numbers
 * live in the regions.  flags: 0 or W4A16_LAUNCH_PDL (then consecutive calls must alternate
 * two workspaces, as for w4a16_gemv_fused). */
int w4a16_gemv_allgather(const uint8_t* packed, const void* scale, int scale_dtype, int group,
                         const void* x, int rows, int cols, int out_dtype, long long row0, int rank,
                         int nranks, void* const* regions, void* workspace, size_t workspace_bytes,
                         unsigned flags, w4a16_stream_t stream);

/* Limit, in nanoseconds, of each wait of w4a16_gemv_allgather on another rank's flags,
 * for the calls made after this one in the process (0 restores the 2 s default; otherwise
 * 1 us .. 60 s, else W4A16_ERR_SHAPE).  A short limit lets a caller that must detect a
 * missing rank quickly (a failure-detection test, a watchdog) get the error code sooner. */
int w4a16_tp_set_peer_wait_ns(unsigned long long ns);

/* ---------------------------------------------------------------------------
 * One-kernel decode step of a Llama-architecture model (no counterpart in the reference,
 * whose end-to-end decode runs the Hugging Face model with its GEMV swapped into every
 * Linear: benchmarks/end_to_end.py:24-42).  One persistent launch per token runs every
 * layer's RMSNorm + QKV GEMV, rotary + KV-cache write + attention, output GEMV + residual,
 * RMSNorm + gate|up GEMV, SwiGLU + down GEMV + residual, then the final norm and the head,
 * with grid-wide barriers between the phases; all projections are int4 with group-128
 * fp32 scales on the interleaved packing.
 * ------------------------------------------------------------------------- */

/* One projection: packed uint8 [rows][cols/2] and fp32 scales [rows][cols/128], both
 * 16-byte aligned device memory. */
typedef struct {
  const uint8_t* packed;
  const float* scale;
} w4a16_g128_weight;

/* A model.  The arrays are host arrays of `layers` entries (read by
 * w4a16_decode_plan_create only); every pointer they hold, and every other pointer, is
 * device memory that must stay valid while the plan is used.
 *   qkv      rows (heads + 2 kv_heads) * head_dim (q | k | v), cols hidden
 *   o        rows hidden, cols heads * head_dim
 *   gate_up  rows 2 * intermediate, cols hidden: gate | up (gate_up_interleaved 0), or gate and
 *            up interleaved in blocks of 8 rows (gate_up_interleaved 8: rows 16k..16k+7 are gate
 *            rows 8k..8k+7, rows 16k+8..16k+15 the matching up rows), which lets the step apply
 *            SwiGLU in the projection's epilogue instead of in the next phase
 *   down     rows hidden, cols intermediate
 *   lm_head  rows vocab, cols hidden
 *   norm_*   fp32 [hidden] RMSNorm weights; embed fp16 [vocab][hidden];
 *   rope_cos, rope_sin  fp32 [max_len][head_dim] rotate-half tables.
 * Limits: head_dim 64; hidden, intermediate and heads * 64 multiples of 1024; hidden at most
 * 4096, intermediate and heads * 64 at most 8192; heads a multiple of kv_heads, at most 8
 * query heads per kv head (Llama-3.2-1B: 2048, 8192, 32 x 64, 4 per kv head). */
typedef struct {
  int layers, hidden, intermediate, heads, kv_heads, head_dim, vocab, max_len;
  float eps;
  const w4a16_g128_weight* qkv;
  const w4a16_g128_weight* o;
  const w4a16_g128_weight* gate_up;
  const w4a16_g128_weight* down;
  const float* const* norm_attn;
  const float* const* norm_mlp;
  w4a16_g128_weight lm_head;
  const float* norm_final;
  const void* embed;
  const float* rope_cos;
  const float* rope_sin;
  int gate_up_interleaved;
} w4a16_llama_desc;

typedef struct w4a16_decode_plan_st* w4a16_decode_plan;

/* Builds the step's tables (tensor maps of every projection) and allocates its scratch on
 * the current device (cudaMalloc; it synchronises the device).  One plan per model and
 * device; free it with w4a16_decode_plan_destroy. */
int w4a16_decode_plan_create(const w4a16_llama_desc* desc, w4a16_decode_plan* plan);
int w4a16_decode_plan_destroy(w4a16_decode_plan plan);

/* One decode step for the token *token at position *pos (device int64 scalars, read by the
 * kernel, so a CUDA graph can replay the step with new values): writes the rotated key and
 * the value of every layer into the caches at pos (fp16 [layers][kv_heads][max_len][64]
 * each) and the logits (fp32 [vocab]).  A pos outside [0, max_len) or a token outside
 * [0, vocab) writes no cache row and gives NaN logits.  Steps of one plan share its scratch:
 * order them on one stream.  Every wait in the kernel is bounded: a wait that runs out sets
 * the device error word (w4a16_read_device_error: 1 weight copy, 3 grid barrier). */
int w4a16_decode_step(w4a16_decode_plan plan, const int64_t* token, const int64_t* pos,
                      void* k_cache, void* v_cache, float* logits, w4a16_stream_t stream);

/* Timeline of the decode step, for finding where a step's time goes.  enable != 0 makes the
 * following steps record %globaltimer (ns) per CTA: entry cta the start, grid + cta the end,
 * 2 grid + cta the moment the first phase's input vector is in place, then for barrier
 * b = 1..5*layers the arrival (3b*grid + cta), the departure ((3b+1)*grid + cta) and the
 * moment the next phase's input is in place ((3b+2)*grid + cta; the attention phase stamps
 * its start); *count receives the number of entries.  With host != NULL
 * (capacity >= *count) the last step's record is copied out (synchronises the stream).
 * enable == 0 stops recording and frees the buffer. */
int w4a16_decode_plan_timeline(w4a16_decode_plan plan, int enable, unsigned long long* host,
                               size_t capacity, size_t* count, w4a16_stream_t stream);

/* Bytes of workspace that let w4a16_gemv balance its work across warps (stream-K)
 * for this batch size; independent of rows and cols (about 0.5 MiB per activation
 * row, at most 16 of them per pass). */
size_t w4a16_gemv_workspace_bytes(int batch, int rows, int cols);

/* No counterpart in the reference.  The same product as w4a16_gemv (interleaved
 * packing, one activation vector, fp32 out, no bias) for callers that cannot
 * allocate device memory — a runtime that fixes its memory plan at start-up, or a
 * plugin interface that passes only input and output buffers.  Split-K scratch comes
 * from a 4 MiB array inside the library (one per GPU that loads it, kept until exit),
 * so nothing is allocated.  The scratch a call needs (w4a16_gemv_workspace_bytes(1,
 * rows, cols), about 0.5 MiB) does not grow with the matrix; a call needing more than
 * 4 MiB would get W4A16_ERR_WORKSPACE with nothing run.  The first call on a device looks up the
 * array's address (again after the device's current context changes); make it before any
 * stream capture.  All calls share the array: calls that overlap on the GPU race, so order
 * them on one stream. */
int w4a16_gemv_noalloc(const uint8_t* packed, const void* scale, int scale_dtype, int group,
                       const void* x, int rows, int cols, float* out, w4a16_stream_t stream);

/* out[r][k] = fp16( fp32(q[r][k]) * fp32(scale(r, k)) ), fp16 [rows][cols], one
 * round-to-nearest per step: bit-identical to (q.float() * scale_expanded).half()
 * computed from the reference's dequant formula (src/w4a16/kernels.py:94-101). */
int w4a16_dequant(const uint8_t* packed, int packing, const void* scale, int scale_dtype,
                  int group, int rows, int cols, void* out, w4a16_stream_t stream);

/* Quantise and pack on the GPU in one launch (the reference does this in torch on
 * the host: quantize_int4_symmetric / quantize_int4_group, src/w4a16/kernels.py:47-60,
 * then pack_int4 / pack_int4_interleaved, :64-91).  w is fp32 or fp16 [rows][cols];
 * scale = max|w| / 7 per row (group 0) or per 128 columns (group 128), computed in
 * fp32; q = clamp(round_half_even(w / scale), -8, 7); an all-zero row or group gets
 * scale 0 and codes 0.  Codes and fp32 scales are bit-identical to the reference's
 * for fp32 input.  packed uint8 [rows][cols/2]; scale fp32 or fp16. */
int w4a16_quantize_pack(const void* w, int w_dtype, int rows, int cols, int group, int packing,
                        uint8_t* packed, void* scale, int scale_dtype, w4a16_stream_t stream);

/* Many activation rows (prefill) on the tensor cores (tcgen05, accumulators in TMEM):
 *   y[m][n] = sum_k x[m][k] * w16[n][k] (+ bias[n]),  w16 = fp16(fp32(q[n][k]) * scale(n, k))
 * w16 is w4a16_dequant's weight, bit for bit, formed in shared memory only; the sums are fp32.
 * The reference runs every call with more than one activation row through F.linear on fp16
 * weights (src/w4a16/kernels.py:120-121); this replaces dequantise-then-GEMM for a caller that
 * keeps no dense copy.  packed uint8 [N][K/2], interleaved packing only, 16-byte aligned;
 * scale fp32 [N] (group 0) or [N][K/128] (group 128); x fp16 [M][K], 16-byte aligned; bias fp32
 * [N] or NULL; y fp32 or fp16 [M][N].  K a multiple of 64 (of 128 with group 128), M, N >= 1,
 * any M and N (ragged tiles are masked).  One CTA per 128 x 128 or 128 x 256 output tile.
 * workspace (optional, 256-byte aligned, zero-filled once; NULL or smaller than
 * w4a16_gemm_workspace_bytes(M, N, K) means no split): when the tiles are fewer than the SMs,
 * K is split across CTAs and the last CTA of each tile sums the fp32 partial tiles in a fixed
 * order (results do not depend on which finishes last); the kernel leaves the workspace's
 * counters zeroed again, except after w4a16_read_device_error reports a non-zero code: then
 * zero-fill it again.  Calls sharing a workspace must be ordered on one stream. */
size_t w4a16_gemm_workspace_bytes(int M, int N, int K);
int w4a16_gemm(const uint8_t* packed, const float* scale, int group, const void* x,
               const float* bias, int M, int N, int K, void* y, int out_dtype, void* workspace,
               size_t workspace_bytes, w4a16_stream_t stream);

/* Reads and clears the error word that kernels set when a bounded wait runs out
 * (0 = none; 1 = a weight copy did not land in time; 2 = another rank's flag did not
 * arrive in time; 3 = a grid barrier of w4a16_decode_step timed out; 4 = a decode plan's
 * shared-memory layout was not aligned, nothing ran; 5 = a pipeline wait of w4a16_gemm
 * gave up, its output tile is incomplete).  Synchronises `stream`.  A non-zero code means some warps returned
 * early: their rows of the output are missing, and a split-K workspace they used may hold
 * non-zero counters, so zero-fill again every workspace used since the previous read
 * (w4a16_gemv_noalloc clears its own on every call). */
int w4a16_read_device_error(int* code, w4a16_stream_t stream);

/* Static text for a status code. */
const char* w4a16_status_string(int status);

/* Detail of the last failure on the calling thread (empty if none). */
const char* w4a16_last_error_string(void);

/* Library version, major * 10000 + minor * 100 + patch. */
int w4a16_version(void);

#ifdef __cplusplus
}
#endif

#endif /* W4A16_B200_H */
