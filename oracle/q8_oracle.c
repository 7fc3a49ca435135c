/* TEST INFRASTRUCTURE ONLY -- the CPU checker for the Q8_0 W8A8 hot path; see q8_oracle.h.
 *
 * Built by oracle/Makefile with -std=c11 -ffp-contract=off, the reference's own rule (its Makefile builds with
 * -std=c11, which keeps GCC from contracting a*b+c into an FMA), so every float operation rounds exactly where the
 * reference's C source says it does. */
#include "q8_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

int orc_quantize(int8_t *q, float *s, const float *x, int n, int gs) {
  /* src/gemv.c:596-623 */
  int groups = n / gs;
  for (int g = 0; g < groups; g++) {
    const float *xg = x + (size_t)g * gs;
    float wmax = 0.0f;
    for (int i = 0; i < gs; i++) {
      if (!isfinite(xg[i]))
        return -1;
      float a = fabsf(xg[i]);
      if (a > wmax)
        wmax = a;
    }
    float scale = wmax / 127.0f;
    s[g] = scale;
    for (int i = 0; i < gs; i++) {
      float v = scale == 0.0f ? 0.0f : xg[i] / scale;
      q[(size_t)g * gs + i] = (int8_t)roundf(fmaxf(-127.0f, fminf(127.0f, v)));
    }
  }
  return 0;
}

int orc_quantize_rows(int8_t *q, float *s, const float *x, size_t ldx, int m, int n, int gs) {
  /* src/gemm.c:818-830: one k_quantize per row, dense outputs */
  for (int r = 0; r < m; r++)
    if (orc_quantize(q + (size_t)r * n, s + (size_t)r * (n / gs), x + (size_t)r * ldx, n, gs))
      return -1;
  return 0;
}

static int32_t group_dot(const int8_t *a, const int8_t *b, int gs) {
  int32_t acc = 0;
  for (int l = 0; l < gs; l++)
    acc += (int32_t)a[l] * (int32_t)b[l];
  return acc;
}

void orc_group_dots(int32_t *dots, const int8_t *xq, int m, int k, int gs, const int8_t *wq, size_t ldw, int n) {
  int groups = k / gs;
  for (int g = 0; g < groups; g++)
    for (int r = 0; r < m; r++)
      for (int c = 0; c < n; c++)
        dots[((size_t)g * m + r) * n + c] =
            group_dot(xq + (size_t)r * k + (size_t)g * gs, wq + (size_t)c * ldw + (size_t)g * gs, gs);
}

void orc_gemv_scalar(float *out, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, size_t ld,
                     int n, int d, int gs) {
  /* src/gemv.c:426-436 */
  size_t scale_ld = ld / (size_t)gs;
  for (int r = 0; r < d; r++) {
    const int8_t *wr = wq + (size_t)r * ld;
    const float *sr = ws + (size_t)r * scale_ld;
    float val = 0.0f;
    for (int j = 0; j <= n - gs; j += gs) {
      int32_t ival = group_dot(xq + j, wr + j, gs);
      val += ((float)ival) * sr[j / gs] * xs[j / gs];
    }
    out[r] = val;
  }
}

float orc_silu_gate(float value, float gate) {
  /* src/gemv.c:246-250 */
  value *= (1.0f / (1.0f + expf(-value)));
  return value * gate;
}

static float amx_order_dot(const int8_t *x, const float *xs, const int8_t *w, const float *ws, int k, int gs) {
  /* src/gemm.c:564-608: out = 0, then per group out = fmaf((float)d * x, scale, out) */
  float acc = 0.0f;
  for (int g = 0; g < k / gs; g++) {
    int32_t d = group_dot(x + (size_t)g * gs, w + (size_t)g * gs, gs);
    float t = (float)d * xs[g];
    acc = fmaf(t, ws[g], acc);
  }
  return acc;
}

void orc_gemm_amx_order(float *c, int ldc, const int8_t *xq, const float *xs, int m, int k, int gs, const int8_t *wq,
                        const float *ws, const int8_t *w3q, const float *w3s, size_t ldw, int n, int kind) {
  int groups = k / gs;
  size_t ws_ld = ldw / (size_t)gs;
  for (int r = 0; r < m; r++)
    for (int j = 0; j < n; j++) {
      const int8_t *x = xq + (size_t)r * k;
      const float *sx = xs + (size_t)r * groups;
      float sum = amx_order_dot(x, sx, wq + (size_t)j * ldw, ws + (size_t)j * ws_ld, k, gs);
      float *out = c + (size_t)r * ldc + j;
      /* src/gemm.c:976-983 */
      if (kind == ORC_ADD)
        *out += sum;
      else if (kind == ORC_SWIGLU)
        *out = orc_silu_gate(sum, amx_order_dot(x, sx, w3q + (size_t)j * ldw, w3s + (size_t)j * ws_ld, k, gs));
      else
        *out = sum;
    }
}

void orc_rmsnorm_scalar(float *o, const float *x, const float *w, int size, float eps) {
  /* src/kernels.c:8-21 */
  float ss = 0.0f;
  for (int j = 0; j < size; j++)
    ss += x[j] * x[j];
  ss /= size;
  ss += eps;
  ss = 1.0f / sqrtf(ss);
  for (int j = 0; j < size; j++)
    o[j] = w[j] * (ss * x[j]);
}

/* _mm512_reduce_add_ps as GCC defines it (avx512fintrin.h __MM512_REDUCE_OP): upper 256 + lower 256, upper 128 +
 * lower 128, then lanes {0,1} + {2,3}, then lane 0 + lane 1. */
static float reduce16(const float *a) {
  float t8[8], t4[4], t2[2];
  for (int i = 0; i < 8; i++)
    t8[i] = a[8 + i] + a[i];
  for (int i = 0; i < 4; i++)
    t4[i] = t8[4 + i] + t8[i];
  t2[0] = t4[0] + t4[2];
  t2[1] = t4[1] + t4[3];
  return t2[0] + t2[1];
}

static float avx512_q8_dot(const int8_t *x, const float *xs, const int8_t *w, const float *ws, int k, int gs) {
  /* dots_q8_body (src/gemv.c:109-139), one row: 16 lanes; per group lane l's int32 sum of bytes 4l..4l+3 of every
   * 64-byte piece (vpdpbusd of |x| and sign(x)*w: the exact signed dot, no int8 value being -128), then
   * acc[l] = fma((float)dot * xs[g], ws[g], acc[l]); the row is the 16 lanes reduced as _mm512_reduce_add_ps. */
  float acc[16];
  memset(acc, 0, sizeof(acc));
  for (int g = 0; g < k / gs; g++) {
    for (int l = 0; l < 16; l++) {
      int32_t d = 0;
      for (int c = 0; c < gs; c += 64)
        for (int b = 0; b < 4; b++) {
          size_t off = (size_t)g * gs + c + 4 * l + b;
          d += (int32_t)x[off] * (int32_t)w[off];
        }
      float t = (float)d * xs[g];
      acc[l] = fmaf(t, ws[g], acc[l]);
    }
  }
  return reduce16(acc);
}

static float portable_q8_dot(const int8_t *x, const float *xs, const int8_t *w, const float *ws, int k, int gs) {
  /* q8_dots' portable loop (src/gemv.c:426-436): val += ((float)ival) * ws * xs per group, ascending */
  float val = 0.0f;
  for (int j = 0; j <= k - gs; j += gs)
    val += ((float)group_dot(x + j, w + j, gs)) * ws[j / gs] * xs[j / gs];
  return val;
}

void orc_gemv_ref_order(float *out, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                        const int8_t *w3q, const float *w3s, size_t ld, int n, int d, int gs, int kind) {
  /* k_matmul_q8 on an AVX-512 host (q8_dots, src/gemv.c:401-416): the AVX-512 body for gs % 64 == 0, else the
   * portable loop; epilogues of q8_range (src/gemv.c:441-480): STORE / PARTIAL write, ADD accumulates, SWIGLU writes
   * silu_gate(dot(w1), dot(w3)). */
  size_t scale_ld = ld / (size_t)gs;
  float (*dot)(const int8_t *, const float *, const int8_t *, const float *, int, int) =
      gs % 64 == 0 ? avx512_q8_dot : portable_q8_dot;
  for (int r = 0; r < d; r++) {
    float sum = dot(xq, xs, wq + (size_t)r * ld, ws + (size_t)r * scale_ld, n, gs);
    if (kind == ORC_ADD)
      out[r] += sum;
    else if (kind == ORC_SWIGLU)
      out[r] = orc_silu_gate(sum, dot(xq, xs, w3q + (size_t)r * ld, w3s + (size_t)r * scale_ld, n, gs));
    else
      out[r] = sum;
  }
}

void orc_gemv_f32_avx512_order(float *out, const float *x, const int8_t *wq, const float *ws, size_t ld, int n, int d,
                               int gs) {
  /* W8A32 (fp32 activations), dots_q8f_body (src/gemv.c:141-180), the reference's path when gs % 16 == 0: per row 16
   * lanes; per group two lane sums ga (columns c + l) and gb (c + 16 + l) over 32-column steps, a 16-column tail into
   * ga, then acc[l] = fma(ga[l] + gb[l], ws[g], acc[l]); the row is the 16 lanes reduced as _mm512_reduce_add_ps. */
  size_t scale_ld = ld / (size_t)gs;
  for (int r = 0; r < d; r++) {
    const int8_t *w = wq + (size_t)r * ld;
    const float *sc = ws + (size_t)r * scale_ld;
    float acc[16];
    memset(acc, 0, sizeof(acc));
    for (int g = 0; g < n / gs; g++) {
      float ga[16], gb[16];
      memset(ga, 0, sizeof(ga));
      memset(gb, 0, sizeof(gb));
      int c = 0;
      for (; c + 32 <= gs; c += 32) {
        size_t off = (size_t)g * gs + c;
        for (int l = 0; l < 16; l++) {
          ga[l] = fmaf((float)w[off + l], x[off + l], ga[l]);
          gb[l] = fmaf((float)w[off + 16 + l], x[off + 16 + l], gb[l]);
        }
      }
      for (; c < gs; c += 16) {
        size_t off = (size_t)g * gs + c;
        for (int l = 0; l < 16; l++)
          ga[l] = fmaf((float)w[off + l], x[off + l], ga[l]);
      }
      for (int l = 0; l < 16; l++)
        acc[l] = fmaf(ga[l] + gb[l], sc[g], acc[l]);
    }
    out[r] = reduce16(acc);
  }
}

void orc_gemv_f32_scalar(float *out, const float *x, const int8_t *wq, const float *ws, size_t ld, int n, int d,
                         int gs) {
  /* W8A32 on q8_dots' portable loop (src/gemv.c:427-436): per group the products summed in column order, then
   * val += group * ws (no fused multiply-add: the reference builds without -march). */
  size_t scale_ld = ld / (size_t)gs;
  for (int r = 0; r < d; r++) {
    const int8_t *w = wq + (size_t)r * ld;
    float val = 0.0f;
    for (int j = 0; j <= n - gs; j += gs) {
      float group = 0.0f;
      for (int k = 0; k < gs; k++)
        group += (float)w[j + k] * x[j + k];
      val += group * ws[(size_t)r * scale_ld + j / gs];
    }
    out[r] = val;
  }
}

void orc_rmsnorm_avx512_order(float *o, const float *x, const float *w, int size, float eps) {
  /* src/kernels_simd.c:136-161 */
  float a[4][16];
  memset(a, 0, sizeof(a));
  int j = 0;
  for (; j + 64 <= size; j += 64)
    for (int v = 0; v < 4; v++)
      for (int l = 0; l < 16; l++)
        a[v][l] = fmaf(x[j + 16 * v + l], x[j + 16 * v + l], a[v][l]);
  for (; j < size; j += 16)
    for (int l = 0; l < 16 && j + l < size; l++)
      a[0][l] = fmaf(x[j + l], x[j + l], a[0][l]);
  float sum[16];
  for (int l = 0; l < 16; l++)
    sum[l] = (a[0][l] + a[1][l]) + (a[2][l] + a[3][l]);
  float ss = reduce16(sum);
  ss /= size;
  ss += eps;
  ss = 1.0f / sqrtf(ss);
  for (j = 0; j < size; j++)
    o[j] = w[j] * (ss * x[j]);
}

static float rope_frequency(int j, int head_dim, float theta, int rope_type, float factor, float low, float high,
                            int original) {
  /* src/kernels.c:49-60 */
  float freq = 1.0f / powf(theta, (float)j / (float)head_dim);
  if (rope_type == 1) {
    float wavelength = 6.2831853071795864769f / freq;
    if (wavelength > original / low)
      freq /= factor;
    else if (wavelength >= original / high) {
      float smooth = (original / wavelength - low) / (high - low);
      freq = (1 - smooth) * freq / factor + smooth * freq;
    }
  }
  return freq;
}

void orc_rope_table(float *table, int position, int head_dim, float theta, int rope_type, float factor, float low,
                    float high, int original) {
  /* src/kernels_simd.c:194-201 */
  for (int j = 0; j < head_dim; j += 2) {
    float angle = position * rope_frequency(j, head_dim, theta, rope_type, factor, low, high, original);
    float c = cosf(angle), s = sinf(angle);
    table[j] = table[j + 1] = c;
    table[head_dim + j] = -s;
    table[head_dim + j + 1] = s;
  }
}

void orc_rope_apply(float *q, float *k, const float *table, int n_heads, int n_kv_heads, int head_dim) {
  /* src/kernels_simd.c:210-227 */
  const float *sines = table + head_dim;
  for (int h = 0; h < n_heads; h++)
    for (int j = 0; j < head_dim; j += 2) {
      float c = table[j], s = sines[j + 1];
      int i = h * head_dim + j;
      float a = q[i], b = q[i + 1];
      q[i] = a * c - b * s;
      q[i + 1] = a * s + b * c;
      if (h < n_kv_heads) {
        a = k[i];
        b = k[i + 1];
        k[i] = a * c - b * s;
        k[i + 1] = a * s + b * c;
      }
    }
}

static uint64_t orc_mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

void orc_random_q8(int8_t *q, float *s, size_t row0, size_t rows, size_t cols, int gs, uint64_t seed,
                   uint64_t tensor, float std) {
  /* Box-Muller pairs: elements 2i and 2i + 1 of a row share one hash pair (r cos t, r sin t). */
  float *row = malloc((cols + 1) * sizeof(float));
  if (!row)
    return;
  for (size_t r = 0; r < rows; r++) {
    for (size_t c = 0; c < cols; c += 2) {
      uint64_t h1 = orc_mix64(seed ^ orc_mix64(tensor * 0x9E3779B97F4A7C15ull + ((row0 + r) * cols + c) / 2));
      uint64_t h2 = orc_mix64(h1 + 0x632BE59BD9B4E019ull);
      float u1 = ((float)(h1 >> 40) + 1.0f) * (1.0f / 16777217.0f), u2 = (float)(h2 >> 40) * (1.0f / 16777216.0f);
      float radius = std * sqrtf(-2.0f * logf(u1)), angle = 6.2831853f * u2;
      row[c] = radius * cosf(angle);
      row[c + 1] = radius * sinf(angle);
    }
    orc_quantize(q + r * cols, s + r * (cols / gs), row, (int)cols, gs);
  }
  free(row);
}

/* ---- attention (src/attention.c), head-major K/V cache [n_kv][seq][hd] ------------------------------------------ */

float orc_exp512(float x) {
  /* exp512 (src/kernels_internal.h:62-76), one lane: clamp to [-87.33654, 88.72283], n = round-to-nearest-even of
   * x * log2(e), r = x - n * ln2 in two fused steps (ln2 split as 0.693359375 - 2.12194440e-4), a degree-6 Horner
   * polynomial in fused steps, y * r^2 + (r + 1), times 2^n. */
  x = fminf(fmaxf(x, -87.33654f), 88.72283f);
  float n = nearbyintf(x * 1.44269504088896341f);
  float r = fmaf(-n, 0.693359375f, x);
  r = fmaf(-n, -2.12194440e-4f, r);
  float y = 1.9875691500e-4f;
  y = fmaf(y, r, 1.3981999507e-3f);
  y = fmaf(y, r, 8.3334519073e-3f);
  y = fmaf(y, r, 4.1665795894e-2f);
  y = fmaf(y, r, 1.6666665459e-1f);
  y = fmaf(y, r, 5.0000001201e-1f);
  y = fmaf(y, r * r, r + 1.0f);
  return ldexpf(y, (int)n);
}

int orc_attention_chunks(int positions, int n_kv_heads, int limit, int workers) {
  /* attention_chunks (src/attention.c:516-526) */
  int chunks = (workers + n_kv_heads - 1) / n_kv_heads;
  int longest = (positions + 31) / 32, shortest = (positions + 255) / 256;
  if (chunks > longest)
    chunks = longest;
  if (chunks < shortest)
    chunks = shortest;
  if (chunks > limit)
    chunks = limit;
  return chunks < 1 ? 1 : chunks;
}

static void merge_partials(const float *base, size_t slot, int chunks, int hd, float *o) {
  /* merge_chunks (src/attention.c:664-682); partials with sum 0 and max -FLT_MAX are skipped */
  float max_val = base[hd];
  for (int c = 1; c < chunks; c++)
    if (base[c * slot + hd] > max_val)
      max_val = base[c * slot + hd];
  float sum = 0.0f;
  memset(o, 0, (size_t)hd * sizeof(float));
  for (int c = 0; c < chunks; c++) {
    const float *chunk = base + c * slot;
    if (chunk[hd + 1] == 0.0f && chunk[hd] == -FLT_MAX)
      continue;
    float weight = expf(chunk[hd] - max_val);
    sum += weight * chunk[hd + 1];
    for (int i = 0; i < hd; i++)
      o[i] += weight * chunk[i];
  }
  for (int i = 0; i < hd; i++)
    o[i] /= sum;
}

static void split_chunk(const float *q, const float *K, const float *V, int hd, int t0, int t1, float *a, float *o) {
  /* attention_chunk_avx512 (src/attention.c:40-105), one head over positions [t0, t1) of its KV head's rows: 16-lane
   * FMA scores over the head's 16-float vectors, _mm512_reduce_add_ps, / sqrtf(hd); the max; exp512 of score - max;
   * lane l of the exp-sum takes positions t0 + 16 i + l; P.V as one FMA chain per output element over the positions. */
  int vectors = (hd + 15) / 16;
  float divisor = sqrtf((float)hd);
  for (int t = t0; t < t1; t++) {
    float lanes[16];
    memset(lanes, 0, sizeof(lanes));
    for (int v = 0; v < vectors; v++)
      for (int l = 0; l < 16 && 16 * v + l < hd; l++)
        lanes[l] = fmaf(q[16 * v + l], K[(size_t)t * hd + 16 * v + l], lanes[l]);
    a[t - t0] = reduce16(lanes) / divisor;
  }
  float max_val = -FLT_MAX;
  for (int t = t0; t < t1; t++)
    if (a[t - t0] > max_val)
      max_val = a[t - t0];
  float vsum[16];
  memset(vsum, 0, sizeof(vsum));
  for (int t = t0; t < t1; t++) {
    float e = orc_exp512(a[t - t0] - max_val);
    a[t - t0] = e;
    vsum[(t - t0) % 16] += e;
  }
  for (int d = 0; d < hd; d++) {
    float acc = 0.0f;
    for (int t = t0; t < t1; t++)
      acc = fmaf(a[t - t0], V[(size_t)t * hd + d], acc);
    o[d] = acc;
  }
  o[hd] = max_val;
  o[hd + 1] = reduce16(vsum);
}

int orc_attention_decode(float *out, const float *q, const float *kc, const float *vc, int n_heads, int n_kv_heads,
                         int hd, int seq, int position, int workers, int limit) {
  /* attention_decode_split (src/attention.c:760-810) with its team's chunk plan: chunks of attention_chunks, chunk c
   * covering [P c / chunks, P (c + 1) / chunks) of the P = position + 1 positions, merged per head. */
  int positions = position + 1, kv_mul = n_heads / n_kv_heads;
  int chunks = orc_attention_chunks(positions, n_kv_heads, limit, workers);
  size_t slot = (size_t)hd + 2;
  float *part = malloc((size_t)chunks * slot * sizeof(float)), *a = malloc((size_t)positions * sizeof(float));
  if (!part || !a) {
    free(part), free(a);
    return -1;
  }
  for (int h = 0; h < n_heads; h++) {
    int g = h / kv_mul;
    const float *K = kc + (size_t)g * seq * hd, *V = vc + (size_t)g * seq * hd;
    for (int c = 0; c < chunks; c++) {
      int t0 = (int)((long long)positions * c / chunks), t1 = (int)((long long)positions * (c + 1) / chunks);
      split_chunk(q + (size_t)h * hd, K, V, hd, t0, t1, a, part + c * slot);
    }
    merge_partials(part, slot, chunks, hd, out + (size_t)h * hd);
  }
  free(part), free(a);
  return 0;
}

static void tiled_chunk(const float *q, const float *K, const float *V, int hd, int t0, int t1, int visible,
                        float *o) {
  /* attention_tiled_avx512 (src/attention.c:245-334), one query vector over chunk [t0, t1) of which it sees positions
   * below `visible`: q scaled by 1 / sqrtf(hd) once; per tile of 32 positions from t0, scores as one FMA chain over the
   * head's elements in order; when the tile's maximum exceeds the running one, the sum and the accumulator are scaled
   * by exp512(old - new); probabilities exp512(score - max); the tile's sum is lanes j and 16 + j added, then
   * _mm512_reduce_add_ps, added to the running sum; P.V as one FMA chain per element over the tile's positions. */
  float scale = 1.0f / sqrtf((float)hd);
  float qs[256], acc[256], m = -FLT_MAX, l = 0.0f;
  for (int d = 0; d < hd; d++)
    qs[d] = q[d] * scale, acc[d] = 0.0f;
  int end = t1 < visible ? t1 : visible;
  if (end <= t0) {
    memset(o, 0, (size_t)hd * sizeof(float));
    o[hd] = -FLT_MAX;
    o[hd + 1] = 0.0f;
    return;
  }
  for (int t = t0; t < end; t += 32) {
    int n = end - t < 32 ? end - t : 32;
    float s[32], e[32];
    for (int j = 0; j < n; j++) {
      float a = 0.0f;
      for (int d = 0; d < hd; d++)
        a = fmaf(qs[d], K[(size_t)(t + j) * hd + d], a);
      s[j] = a;
    }
    float tile_max = -FLT_MAX;
    for (int j = 0; j < n; j++)
      if (s[j] > tile_max)
        tile_max = s[j];
    if (tile_max > m) {
      float alpha = orc_exp512(m - tile_max);
      l *= alpha;
      for (int d = 0; d < hd; d++)
        acc[d] *= alpha;
      m = tile_max;
    }
    float lanes[16];
    for (int j = 0; j < 32; j++)
      e[j] = j < n ? orc_exp512(s[j] - m) : 0.0f;
    for (int j = 0; j < 16; j++)
      lanes[j] = e[j] + e[16 + j];
    l += reduce16(lanes);
    for (int j = 0; j < n; j++)
      for (int d = 0; d < hd; d++)
        acc[d] = fmaf(e[j], V[(size_t)(t + j) * hd + d], acc[d]);
  }
  for (int d = 0; d < hd; d++)
    o[d] = acc[d];
  o[hd] = m;
  o[hd + 1] = l;
}

int orc_attention_tiled(float *out, const float *q, const float *kc, const float *vc, int n_heads, int n_kv_heads,
                        int hd, int seq, int pos0, int m, int workers, int limit) {
  /* attention_tiled_driver (src/attention.c:1175-1229) for m > 1 rows at positions pos0.. (row r sees pos0 + r + 1
   * positions): rows in blocks of 16 / (query heads per KV head); tiled_plan (src/attention.c:1078-1085) gives each
   * block's chunk length (a multiple of 32) and count from attention_chunks at its last row; every row of the block
   * uses that plan, its chunks merged per head. out and q: m rows of n_heads * hd. */
  int kv_mul = n_heads / n_kv_heads, rblock = 16 / kv_mul < 1 ? 1 : 16 / kv_mul;
  size_t slot = (size_t)hd + 2;
  int max_chunks = orc_attention_chunks(pos0 + m, n_kv_heads, limit, workers);
  float *part = malloc((size_t)(max_chunks + 1) * slot * sizeof(float));
  if (!part || hd > 256)
    return free(part), -1;
  for (int r = 0; r < m; r++) {
    int block = r / rblock, block_end = (block + 1) * rblock < m ? (block + 1) * rblock : m;
    int positions = pos0 + block_end;
    int wanted = orc_attention_chunks(positions, n_kv_heads, limit, workers);
    int len = ((positions + wanted - 1) / wanted + 31) / 32 * 32, chunks = (positions + len - 1) / len;
    for (int h = 0; h < n_heads; h++) {
      int g = h / kv_mul;
      const float *K = kc + (size_t)g * seq * hd, *V = vc + (size_t)g * seq * hd;
      for (int c = 0; c < chunks; c++) {
        int t0 = c * len, t1 = (c + 1) * len < positions ? (c + 1) * len : positions;
        tiled_chunk(q + ((size_t)r * n_heads + h) * hd, K, V, hd, t0, t1, pos0 + r + 1, part + c * slot);
      }
      merge_partials(part, slot, chunks, hd, out + ((size_t)r * n_heads + h) * hd);
    }
  }
  free(part);
  return 0;
}
