/* TEST INFRASTRUCTURE ONLY -- the CPU checker for the Q8_0 W8A8 hot path; see q8_oracle.h.
 *
 * Built by oracle/Makefile with -std=c11 -ffp-contract=off, the reference's own rule (its Makefile builds with
 * -std=c11, which keeps GCC from contracting a*b+c into an FMA), so every float operation rounds exactly where the
 * reference's C source says it does. */
#include "q8_oracle.h"

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
