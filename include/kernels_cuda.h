/* B200 (sm_100a) backend of llama3.x.c's Q8_0 W8A8 kernel API: the C-ABI of libllama3x_cuda.so.
 *
 * Each entry point keeps the name, argument order and meaning of the reference function it replaces (cited below as
 * include/kernels.h:LINE or include/gemm.h:LINE of LucianCrainic/llama3.x.c), with two differences:
 *   1. Every pointer is a DEVICE pointer (CUDA global memory). Work is queued on the calling thread's stream
 *      (kernels_set_stream; the legacy default stream until then) and the call returns before the GPU finishes;
 *      kc_status() waits for the stream and reports errors the kernels found (non-finite activations, timeouts).
 *   2. "Team" becomes "stream": kernels_set_stream replaces kernels_set_team / kernels_set_thread_team
 *      (include/kernels.h:24-28).
 * Errors keep the reference's behaviour by default: invalid arguments and CUDA failures print the message and exit(1),
 * as fail() does (include/runtime.h:29). kc_set_fail_mode(KC_FAIL_RETURN) instead records the message
 * (kc_last_error) and returns without queuing work, for callers that cannot lose the process.
 *
 * Weight layout is the checkpoint's: values row-major [rows][ld] int8 (ld a multiple of gs), scales [rows][ld / gs]
 * fp32. Weight values, weight scales and activations passed to the GEMV/GEMM must be 16-byte aligned, and ld / gs a
 * multiple of 4 (cudaMalloc'd buffers with the reference's shapes satisfy this). The fast kernels take group sizes
 * 64, 128, 256 (the checkpoints use 64); other group sizes take a slower general kernel in the reference's portable
 * order.
 * W8A32 (K8Input.q == NULL, fp32 activations in f) runs on every k_matmul_q8* entry point, bitwise the reference's
 * AVX-512 kernel (dots_q8f_body, src/gemv.c:141-180) when gs % 16 == 0 and its portable loop otherwise. */
#ifndef LLAMA3X_KERNELS_CUDA_H
#define LLAMA3X_KERNELS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* include/kernels.h:101-109 */
typedef struct {
  const int8_t *q;
  const float *s;
} K8Weight;
typedef struct {
  const int8_t *q;
  const float *s;
  const float *f;
} K8Input;

/* include/kernels.h:84 */
typedef enum { K_STORE, K_ADD, K_PARTIAL, K_SWIGLU } KernelEpilogue;
/* include/gemm.h:15-20 */
typedef enum { GEMM_STORE, GEMM_ADD, GEMM_SWIGLU, GEMM_PARTIAL } GemmKind;
enum { GEMM_MAX_SEGMENTS = 3 }; /* include/gemm.h:32 */

/* include/gemm.h:118-125. pw / pw3 (the reference's AMX-packed copies) are ignored: the tensor-core path reads the
 * checkpoint's row-major values directly through TMA. */
typedef struct {
  float *c;
  int ldc;
  K8Weight w, w3;
  const int8_t *pw, *pw3;
  int n;
  GemmKind kind;
} GemmQ8Segment;

/* include/gemm.h:126, extended with this backend's two kernels. PORTABLE / AVX512 / AMX are CPU rungs and are not
 * compiled in here (k_gemm_q8_backend_test returns 0 for them, as the reference does for a rung it lacks). */
typedef enum {
  Q8_GEMM_PORTABLE,
  Q8_GEMM_AVX512,
  Q8_GEMM_AMX,
  Q8_GEMM_GPU_DP4A = 16,   /* the row kernel (decode GEMV, the reference's AVX-512 / portable order), one launch per
                              activation row */
  Q8_GEMM_GPU_TCGEN05 = 17 /* tcgen05 int8 MMA with TMEM accumulators, fed by TMA (the AMX-INT8 order) */
} Q8GemmBackend;

/* ---- set-up (include/kernels.h:16-31) ---------------------------------------------------------------------------- */
void kernels_init(void);                /* binds the library to the current CUDA device */
const char *kernels_name(void);         /* "sm_100a" after kernels_init, NULL before */
void kernels_set_stream(void *stream);  /* cudaStream_t for this thread's kernels; NULL = legacy default stream */
/* Programmatic dependent launch for the GEMV/GEMM (on by default): their weight streams start while the previous
 * kernel in the stream finishes. No reference counterpart (a CPU team has no launch latency to hide). */
void kernels_set_pdl(int on);
/* The reference's CPU worker-team set-up and teardown (include/kernels.h:29-30): the GPU has no team to build, so both
 * do nothing; they exist so that callers written for the reference link unchanged. */
void kernels_backend_init(void);
void kernels_backend_free(void);

/* ---- error handling (runtime.h fail() analogue) ----------------------------------------------------------------- */
enum { KC_FAIL_EXIT = 0, KC_FAIL_RETURN = 1 };
void kc_set_fail_mode(int mode);
const char *kc_last_error(void); /* last recorded message, "" if none; cleared by kc_clear_error */
void kc_clear_error(void);
/* Waits for this thread's stream, then returns and clears the device error bits (1 = non-finite activation in a
 * quantizer, 2 = a bounded wait timed out, 4 = bad arguments), or -1 for a CUDA error. In KC_FAIL_EXIT mode a
 * nonzero result fails like the reference ("nonfinite activation during INT8 quantization"). */
int kc_status(void);
/* Applies the fail() policy to a message from a caller of this library (the GPU engine): exit under KC_FAIL_EXIT,
 * else record it for kc_last_error. */
void kc_fail_message(const char *message);
/* Kernels this library has launched in this process since it was loaded, counted at each successful launch call (no
 * counterpart in the reference). A CUDA-graph replay launches its captured kernels without calling in here. */
unsigned long long kc_launch_count(void);

/* ---- quantizer (include/kernels.h:110, include/gemm.h:130) ------------------------------------------------------- */
void k_quantize(int8_t *q, float *s, const float *x, int n, int gs);
void k_quantize_rows(int8_t *q, float *s, const float *x, size_t ldx, int m, int n, int gs);

/* ---- decode GEMV (include/kernels.h:111-122) --------------------------------------------------------------------- */
/* Bitwise the reference's k_matmul_q8 on an AVX-512 host (q8_dots, src/gemv.c:401-438): dots_q8_body's 16-lane order
 * for gs % 64 == 0, the portable loop otherwise; W8A32 (x->q NULL) in dots_q8f_body's order or the portable loop. */
void k_matmul_q8(float *out, const K8Input *x, K8Weight w, int n, int d, int gs);
void k_matmul_q8_add(float *out, const K8Input *x, K8Weight w, int n, int d, int gs);
void k_matmul_q8_qkv(float *q, float *k, float *v, const K8Input *x, K8Weight wq, K8Weight wk, K8Weight wv, int n,
                     int dq, int dkv, int gs);
void k_matmul_q8_swiglu(float *out, const K8Input *x, K8Weight w1, K8Weight w3, int n, int d, int gs);
void k_matmul_q8_ld(float *out, const K8Input *x, const K8Weight *w, size_t ld, int n, int d, int gs, int kind);
void k_matmul_q8_swiglu_ld(float *out, const K8Input *x, const K8Weight *w1, const K8Weight *w3, size_t ld, int n,
                           int d, int gs);
/* Member `worker` of `workers`' share of k_matmul_q8_ld (include/kernels.h:86-95, 119-120): output rows
 * [d * worker / workers, d * (worker + 1) / workers), the reference's static Q8 split (src/gemv.c:488-495); the
 * members' shares together are the full product, bitwise. `claim` is ignored, as the reference ignores it for Q8.
 * `done`, when not NULL, is called as done(done_ctx, r0, r1) once the share's rows are in memory (this call waits for
 * the stream), so a caller can start on those rows. */
typedef void (*RowsDoneFn)(void *ctx, int r0, int r1);
#ifdef __cplusplus
typedef int kc_atomic_int; /* the reference's atomic_int, only passed through */
#else
#include <stdatomic.h>
typedef atomic_int kc_atomic_int;
#endif
void k_matmul_q8_ld_worker(float *out, const K8Input *x, const K8Weight *w, size_t ld, int n, int d, int gs, int kind,
                           int worker, int workers, kc_atomic_int *claim, RowsDoneFn done, void *done_ctx);

/* The decode GEMV with its input prepared inside the kernel (no reference counterpart): x holds n fp32 activations,
 * RMS-normalized with `weight` and `epsilon` first when weight is not NULL (k_rmsnorm_q8_rows' arithmetic), then
 * quantized in gs-groups (k_quantize's rule) by every CTA into its own shared memory, while the first weight stages
 * stream in. Bitwise the pair k_rmsnorm_q8_rows (or k_quantize) + k_matmul_q8*, in one launch. The 1-3 segments share
 * one kind: GEMM_STORE, GEMM_ADD, GEMM_PARTIAL (rows `n` of c from w) or GEMM_SWIGLU (one segment, w and w3); weight
 * rows have stride ld. gs 64, 128 or 256. */
typedef struct KernelTail KernelTail;
/* `tail` (may be NULL) as for k_matmul_q8_tail below. */
void k_matmul_q8_fused(const float *x, const float *weight, float epsilon, size_t ld, int n, int gs,
                       const GemmQ8Segment *segments, int count, const KernelTail *tail);

/* The decode GEMV followed by work its last CTA does once, after every CTA's outputs are in memory (no reference
 * counterpart): a kernel boundary saved between a GEMV and the small step the next one needs.
 *   K_TAIL_QUANTIZE:        k_quantize(q, s, x, n, gs), e.g. of the SwiGLU output the GEMV just wrote;
 *   K_TAIL_NORM_QUANTIZE:   k_rmsnorm_q8_rows(q, s, NULL, x, n, weight, 1, n, epsilon, gs), e.g. of the residual the
 *                           GEMV just added into (the next layer's input);
 *   K_TAIL_ROPE_KV_STORE:   k_rope_kv_store_rows on the three segments' outputs (q, k, v) at *position;
 *   K_TAIL_QUANTIZE_OUTPUT: k_quantize(q, s, c, n, gs) of the GEMV's own output (one GEMM_STORE or GEMM_SWIGLU segment
 *                           of n rows, n % gs == 0, n / gs <= 65536), not by the last CTA but by each CTA for the
 *                           groups its rows complete (a per-group counter), so the quantization adds no serial step.
 * Bitwise the separate kernels. The input is the usual K8Input and the segments share one kind (as
 * k_matmul_q8_fused). Tail GEMVs in flight on two streams of one device at once race on the kernel's completion
 * counters. */
typedef enum {
  K_TAIL_NONE,
  K_TAIL_QUANTIZE,
  K_TAIL_NORM_QUANTIZE,
  K_TAIL_ROPE_KV_STORE,
  K_TAIL_QUANTIZE_OUTPUT
} KernelTailKind;
struct KernelTail {
  KernelTailKind kind;
  const float *x;      /* (NORM_)QUANTIZE: n values, and the RMSNorm weights and epsilon */
  const float *weight;
  float epsilon;
  int8_t *q;
  float *s;
  int n;
  const float *rope_table; /* ROPE_KV_STORE: [seq_len][2 * head_dim], the position in device memory, the caches */
  const int *position;
  float *key_cache, *value_cache;
  int n_heads, n_kv_heads, head_dim, seq_len;
};
void k_matmul_q8_tail(const K8Input *x, size_t ld, int n, int gs, const GemmQ8Segment *segments, int count,
                      const KernelTail *tail);

/* ---- AMX packing helpers (include/gemm.h:55-67, 136-144) ---------------------------------------------------------- */
/* The reference's int8 tile layout for its AMX kernels, produced on the host: rows in tiles of 16, K in quads, both
 * zero-padded (K to 64): dst[((tile * kp / 4 + quad) * 16 + row_in_tile) * 4 + byte] with kp = cols rounded up to 64.
 * The sm_100a GEMM reads the row-major weights through TMA and never these copies (GemmQ8Segment.pw is ignored); the
 * helpers exist so that loaders written for the reference link unchanged and get the same bytes. Host memory. */
size_t s8_vnni_bytes(int rows, int cols);
void pack_s8_vnni(int8_t *dst, const int8_t *w, int rows, int cols, size_t ld);
void pack_s8_vnni_tiles(int8_t *dst, const int8_t *w, int rows, int cols, size_t ld, int first, int last);
typedef struct {
  int8_t *dst;
  const int8_t *w;
  int rows, cols;
  size_t ld;
} PackS8;
void pack_s8_vnni_many(const PackS8 *jobs, int count);

/* ---- batched prefill GEMM (include/gemm.h:130-135) --------------------------------------------------------------- */
/* Shapes the tensor-core kernel takes (gs 64, k % 256 == 0, 16-byte aligned operands, a SwiGLU pair as the only
 * segment) run on it at every row count, in the reference's AMX-INT8 order (amx_q8_chunk, src/gemm.c:554-610), so a
 * row's result never depends on its batch; other shapes run one decode GEMV per row, in the order of the reference's
 * AVX-512 GEMM rung for gs % 64 == 0 (bitwise its GEMV, src/gemm.c:862-899) and of its portable rung otherwise.
 * k_gemm_q8_pick reports the rung for the segments (src/gemm.c:991-1004); it cannot see k or the activations, so a
 * k % 256 != 0 or an unaligned activation pointer still sends k_gemm_q8 to the row rung. The tensor-core path stages the transposed activation scales in one buffer per device that the library
 * grows with cudaMalloc when a call needs more (k_gemm_q8_noalloc uses a fixed array instead). Every call on a device
 * shares that buffer, so calls on one device must not overlap on the GPU: issue them from one stream, as the
 * reference's team_run is not reentrant (include/workers.h:26). */
void k_gemm_q8(const int8_t *xq, const float *xs, int m, int k, int gs, const GemmQ8Segment *segments, int count);
Q8GemmBackend k_gemm_q8_pick(int gs, const GemmQ8Segment *segments, int count);

/* ---- supporting kernels (include/kernels.h:57-68) ---------------------------------------------------------------- */
void k_rmsnorm(float *out, const float *x, const float *weight, int size, float epsilon);
void k_rmsnorm_rows(float *out, const float *x, const float *weight, int rows, int size, float epsilon);
void k_rope_apply(float *q, float *k, const float *table, int n_heads, int n_kv_heads, int head_dim);
void k_rope_apply_rows(float *q, size_t q_stride, float *k, size_t k_stride, const float *table, size_t table_stride,
                       int rows, int n_heads, int n_kv_heads, int head_dim);

/* Fused RMSNorm + quantize: the reference's k_rmsnorm_rows followed by k_quantize_rows (src/tp.c:403-404,
 * src/tp.c:539-540) in one kernel. `out` (the fp32 normalized rows, stride size) may be NULL. Bitwise equal to the
 * pair on the reference's AVX-512 ISA. */
void k_rmsnorm_q8_rows(int8_t *q, float *s, float *out, const float *x, size_t ldx, const float *weight, int rows,
                       int size, float epsilon, int gs);

/* ---- K/V cache and attention (include/kernels.h:126-179) --------------------------------------------------------- */
/* The cache is the reference's head-major layout (LLAMA_KV_LAYOUT=head, its default): one layer's K or V cache is
 * [n_kv_heads][seq_len][head_dim] fp32. AttentionWork holds the split-K partials in device memory (the reference keeps
 * them in host memory); head_dim 32, 64 or 128 with at most 16 query heads per KV head take the fast kernels, other
 * shapes up to head_dim 256 a slower restatement of the same arithmetic. `memory` passed to k_attention_init_rows is
 * device memory of k_attention_bytes_rows bytes (the partials, then 1 KiB of merge tickets that the call zeroes on
 * the library's stream), or NULL to let the call allocate it (k_attention_free releases only what it allocated).
 * One row runs the split decode kernel, which is bitwise the reference's AVX-512 decode attention
 * (attention_chunk_avx512 + merge_chunks, src/attention.c) with the chunk plan of a team of one (256-position
 * chunks); a batch runs the tiled kernel, bitwise its batched attention (attention_tiled_avx512, src/attention.c:233-344,
 * planned as at src/attention.c:1078-1085).
 * `att` is the reference's host scratch and is ignored. AttentionWork has the reference's layout
 * (include/kernels.h:127-132), so a caller compiled against the reference's header passes a struct this library
 * reads field for field: partial (device memory), max_chunks (the 256-position splits of the longest context it
 * serves), n_heads and head_dim (checked against each call), workers (always 1: one GPU does the work of the
 * reference's team), external and capacity (floats of partials in partial). */
typedef struct {
  float *partial;
  int max_chunks, n_heads, head_dim, workers;
  int external;
  size_t capacity;
} AttentionWork;
void k_kv_strides(int n_kv_heads, int head_dim, int seq_len, size_t *pos_stride, size_t *head_base);
void k_kv_store(float *cache, const float *src, size_t src_ld, int pos0, int count, int n_kv_heads, int head_dim,
                int seq_len);
size_t k_attention_bytes_rows(int n_heads, int n_kv_heads, int head_dim, int seq_len, int rows);
void k_attention_init_rows(AttentionWork *work, int n_heads, int n_kv_heads, int head_dim, int seq_len, int rows,
                           void *memory);
void k_attention_free(AttentionWork *work);
void k_attention_kv(float *out, const float *q, const float *key_cache, const float *value_cache, float *att,
                    AttentionWork *work, int n_heads, int n_kv_heads, int head_dim, int seq_len, int position);
void k_attention_batch_kv(float *out, const float *q, const float *key_cache, const float *value_cache, float *att,
                          AttentionWork *work, int n_heads, int n_kv_heads, int head_dim, int seq_len, int pos0, int m);

/* ---- GPU engine steps (no counterpart in the reference, whose engine does these inline on the host) -------------- */
/* Fused k_rope_apply_rows + two k_kv_store calls (src/tp.c:549-556): rows r of q (stride q_ld) and k (stride kv_ld)
 * rotated at position (*position if non-NULL, else pos0) + r with table [seq_len][2 * head_dim] (k_rope_table rows);
 * q rotated in place, rotated k and v (stride kv_ld) stored into the caches. Reading the position from device memory
 * lets a captured decode step replay at every position. */
void k_rope_kv_store_rows(float *q, size_t q_ld, const float *k, const float *v, size_t kv_ld, float *key_cache,
                          float *value_cache, const float *table, const int *position, int pos0, int rows, int n_heads,
                          int n_kv_heads, int head_dim, int seq_len);
/* The decode step's k_rope_kv_store_rows + k_attention_q8_rows (one row, device position) in one launch: q, k, v are
 * the unrotated QKV product of position *position; the queries and the new key are rotated with `table` (row
 * *position) as k_rope_kv_store_rows does, the new K/V row is used directly and written into the caches for later
 * positions, and q is left unrotated. Bitwise the two calls it replaces. The launch before it must write neither
 * *position nor any cache row at or below *position. k_rope_attention_q8_step_ok(n_heads, n_kv_heads, head_dim, gs)
 * tells whether a shape is supported (gs <= 0: without the output quantization); other shapes use the two calls. */
int k_rope_attention_q8_step_ok(int n_heads, int n_kv_heads, int head_dim, int gs);
void k_rope_attention_q8_step(float *out, int8_t *oq, float *os, const float *q, const float *k, const float *v,
                              float *key_cache, float *value_cache, const float *table, AttentionWork *work,
                              int n_heads, int n_kv_heads, int head_dim, int seq_len, const int *position, int gs);
/* k_attention_batch_kv whose output is also quantized for the Wo product (k_quantize_rows fused, src/tp.c:562),
 * oq/os may be NULL; with a device `position` the rows are at *position + r.
 * With a device `position` and one row (the decode step), the kernel reads *position and requests the cache rows
 * below it before it waits on the kernel launched just before it on the stream: that launch must write neither the
 * position word nor any cache row below *position (a decode step's K/V store of row *position itself is fine). */
void k_attention_q8_rows(float *out, int8_t *oq, float *os, const float *q, const float *key_cache,
                         const float *value_cache, AttentionWork *work, int n_heads, int n_kv_heads, int head_dim,
                         int seq_len, const int *position, int pos0, int rows, int gs);
/* x[r][i] = q[tok][i] * s[(tok * dim + i) / gs] for tok = tokens[r] (device), src/tp.c:395-396. */
void k_embed_q8_rows(float *x, const int *tokens, K8Weight embed, int rows, int dim, int gs, int vocab);
void k_add(float *x, const float *y, size_t n); /* x += y */
/* Greedy sampling on the device: folds into *key (which must hold 0 or an earlier key) a 64-bit key whose unsigned
 * maximum over all shards (an NCCL max all-reduce) is the first maximum (sample_argmax, src/sampler.c:9-23);
 * logits[i] has vocabulary index offset + i. */
void k_argmax_key(unsigned long long *key, const float *logits, int n, int offset);
/* token = index in *key; out[*step] = token (out may be NULL); *token = token; ++*step; ++*position; *key = 0. */
void k_greedy_advance(int *out, int *step, int *token, int *position, unsigned long long *key);
/* Seeded N(0, std) benchmark weights quantized like k_quantize: rows [row0, row0 + rows) x columns [col0, col0 + cols)
 * of a [*][full_cols] tensor numbered `tensor`, into q [rows][cols] and s [rows][cols / gs]; every element is a
 * function of (seed, tensor, row, column) only, so a shard equals the same slice of the whole tensor. gs 32..256. */
void k_random_q8(int8_t *q, float *s, int rows, int cols, size_t row0, size_t col0, size_t full_cols,
                 unsigned long long seed, unsigned long long tensor, float std, int gs);
void k_fill(float *x, size_t n, float value);

/* ---- test hooks (include/testing.h:67-69) ------------------------------------------------------------------------ */
/* One named backend; returns 0 when it is not compiled in (the CPU rungs). */
int k_gemm_q8_backend_test(Q8GemmBackend backend, const int8_t *xq, const float *xs, int m, int k, int gs,
                           const GemmQ8Segment *segments, int count);
/* The exact int32 group dots of the tensor-core kernel, dots[(g * m + r) * n + c] (k_gemm_q8_amx_dots_test's layout),
 * from row-major weights wq[n][k] instead of an AMX-packed copy. Returns 0 when unsupported. */
int k_gemm_q8_dots_test(int32_t *dots, const int8_t *xq, int m, int k, int gs, const int8_t *wq, int n);

/* ---- k_gemm_q8 without device allocation (no counterpart in the reference) -------------------------------------- */
/* Same arguments and results as k_gemm_q8, but the tensor-core path stages its transposed activation scales in a
 * fixed array compiled into the library (K_GEMM_Q8_NOALLOC_MAX_SCALES floats, 4 MiB, one per device) instead of a
 * buffer it allocates: (k / gs) * round_up(m, 4) must not exceed that, or the call is rejected. The first call on a
 * device looks the array's address up (cudaGetSymbolAddress, with that device current, under a lock), so make it once
 * during setup, before any stream capture. The address is kept for the life of the process: after cudaDeviceReset
 * the module loads again elsewhere, so do not call this entry point on a device that was reset.
 * Nothing needs to start at zero: every call rewrites the whole part of the array it reads. Calls on one device share
 * the array, so two calls in flight at once (different streams or threads) race; issue them on one stream.
 * Returns 0 on success, -1 when the arguments are rejected (kc_last_error says why, under KC_FAIL_RETURN). */
#define K_GEMM_Q8_NOALLOC_MAX_SCALES (1 << 20)
int k_gemm_q8_noalloc(const int8_t *xq, const float *xs, int m, int k, int gs, const GemmQ8Segment *segments,
                      int count);

#ifdef __cplusplus
}
#endif

#endif
