/* TEST INFRASTRUCTURE ONLY -- never linked into, loaded by, or called from the product path.
 *
 * CPU restatement of the reference's Q8_0 W8A8 hot path (LucianCrainic/llama3.x.c), used by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline leg as the checker. Every function names the reference
 * file:line it restates. Parity is pinned two ways (tests/test_oracle.py):
 *   - against the reference itself, compiled from its own sources into oracle/_ref/ by oracle/Makefile, on seeded
 *     inputs (when oracle/_ref is present);
 *   - against golden vectors under tests/golden/ produced by that compiled reference (tests/golden/make_golden.py),
 *     including the reference test suite's own known-answer quantizer ties (tests/kernels.c:111-116).
 * Functions return 0 on success and a negative code where the reference would call fail(). */
#ifndef Q8_ORACLE_H
#define Q8_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_STORE = 0, ORC_ADD = 1, ORC_PARTIAL = 2, ORC_SWIGLU = 3 };

/* k_quantize (src/gemv.c:589-624): per group max|x| (non-finite input fails), scale = max / 127.0f,
 * q = (int8)roundf(clamp(x / scale, -127, 127)), q = 0 when the scale is 0. Returns -1 on non-finite input. */
int orc_quantize(int8_t *q, float *s, const float *x, int n, int gs);
/* k_quantize_rows (src/gemm.c:818-830): k_quantize per row; row r of x has stride ldx, of q stride n, of s n/gs. */
int orc_quantize_rows(int8_t *q, float *s, const float *x, size_t ldx, int m, int n, int gs);

/* Exact int32 group dots, dots[(g * m + r) * n + c] (the layout of k_gemm_q8_amx_dots_test, src/gemm.c:1043-1066). */
void orc_group_dots(int32_t *dots, const int8_t *xq, int m, int k, int gs, const int8_t *wq, size_t ldw, int n);

/* The scalar GEMV order (q8_dots, src/gemv.c:417-438): val += ((float)ival) * ws * xs per group, ascending. */
void orc_gemv_scalar(float *out, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, size_t ld,
                     int n, int d, int gs);

/* The reference's decode GEMV, k_matmul_q8 on an AVX-512 host (q8_dots, src/gemv.c:401-438): dots_q8_body's 16-lane
 * order for gs % 64 == 0 (per lane an exact int32 sum of bytes 4l..4l+3 of each 64-byte piece, an FMA chain over the
 * groups, then _mm512_reduce_add_ps), the portable loop otherwise; one activation row, d weight rows, with the
 * STORE / ADD / PARTIAL / SWIGLU epilogues (w3q / w3s for SWIGLU). */
void orc_gemv_ref_order(float *out, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                        const int8_t *w3q, const float *w3s, size_t ld, int n, int d, int gs, int kind);

/* The AMX-INT8 order (amx_q8_chunk, src/gemm.c:554-610): acc = fmaf((float)dot * xs, ws, acc) per group, ascending,
 * from acc = 0. C[m][n] for one segment; `kind` applies the epilogue of q8_gemm_chunks (src/gemm.c:963-989):
 * STORE / PARTIAL write, ADD accumulates, SWIGLU writes silu_gate(acc(w), acc(w3)). */
void orc_gemm_amx_order(float *c, int ldc, const int8_t *xq, const float *xs, int m, int k, int gs, const int8_t *wq,
                        const float *ws, const int8_t *w3q, const float *w3s, size_t ldw, int n, int kind);

/* silu_gate (src/gemv.c:246-250). */
/* W8A32 GEMV (fp32 activations x, int8 weights): the reference's AVX-512 order (gs % 16 == 0) and its portable loop. */
void orc_gemv_f32_avx512_order(float *out, const float *x, const int8_t *wq, const float *ws, size_t ld, int n, int d,
                               int gs);
void orc_gemv_f32_scalar(float *out, const float *x, const int8_t *wq, const float *ws, size_t ld, int n, int d, int gs);
float orc_silu_gate(float value, float gate);

/* rmsnorm_eps, the scalar order (src/kernels.c:8-21). */
void orc_rmsnorm_scalar(float *o, const float *x, const float *w, int size, float eps);
/* rmsnorm_avx512 (src/kernels_simd.c:136-161): four 16-lane FMA accumulators over 64-value steps, a masked tail into
 * the first, _mm512_reduce_add_ps of (a0 + a1) + (a2 + a3), then the scalar epilogue. */
void orc_rmsnorm_avx512_order(float *o, const float *x, const float *w, int size, float eps);

/* k_rope_table (src/kernels_simd.c:194-201) with rope_frequency (src/kernels.c:49-60); k_rope_apply scalar
 * (src/kernels_simd.c:203-227). */
void orc_rope_table(float *table, int position, int head_dim, float theta, int rope_type, float factor, float low,
                    float high, int original);
void orc_rope_apply(float *q, float *k, const float *table, int n_heads, int n_kv_heads, int head_dim);

/* The reference's attention on the head-major cache [n_kv_heads][seq][hd] (its default LLAMA_KV_LAYOUT=head), with
 * its team's chunk plan (`workers`, attention_chunks src/attention.c:516-526; `limit` = the work's max_chunks):
 * orc_attention_decode is the split decode (src/attention.c:40-105, 664-682, 760-810) for one row at `position`;
 * orc_attention_tiled the default batched variant (src/attention.c:245-334, 1078-1229) for m > 1 rows from pos0.
 * orc_exp512 is exp512 (src/kernels_internal.h:62-76) on one lane. Return -1 on allocation failure. */
float orc_exp512(float x);
int orc_attention_chunks(int positions, int n_kv_heads, int limit, int workers);
int orc_attention_decode(float *out, const float *q, const float *kc, const float *vc, int n_heads, int n_kv_heads,
                         int hd, int seq, int position, int workers, int limit);
int orc_attention_tiled(float *out, const float *q, const float *kc, const float *vc, int n_heads, int n_kv_heads,
                        int hd, int seq, int pos0, int m, int workers, int limit);

#ifdef __cplusplus
}
#endif

#endif

/* Seeded N(0, std) values by element index (SplitMix64 finalizer feeding Box-Muller in double precision), rows
 * [row0, row0 + rows) of a [*][cols] tensor numbered `tensor`, quantized with orc_quantize's rule into q [rows][cols]
 * and s [rows][cols / gs]. Used to write benchmark-size checkpoints for the reference's CPU engine. */
void orc_random_q8(int8_t *q, float *s, size_t row0, size_t rows, size_t cols, int gs, uint64_t seed,
                   uint64_t tensor, float std);
