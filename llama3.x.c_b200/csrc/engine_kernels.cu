// Per-token kernels of the GPU forward pass (the C11 engine, engine.c): embedding dequantization, RoPE fused with the
// K/V store, GQA attention over the fp32 head-major K/V cache with its output quantized in the same kernel, residual
// add, greedy argmax, and the seeded Q8 generator of the benchmark models.
//
// Reference semantics (LucianCrainic/llama3.x.c):
//  - embedding: x[i] = (float)q[row * dim + i] * s[(row * dim + i) / gs]                  (src/tp.c:395-396)
//  - RoPE from the host-built table (k_rope_table / k_rope_apply, src/kernels_simd.c:194-227), bitwise
//  - K/V cache head-major [kv_head][position][head_dim] (k_kv_store / k_kv_strides, src/attention.c:1415-1432)
//  - attention per head: score_t = (q . k_t) / sqrtf(head_dim), softmax over t <= pos, out = sum_t w_t v_t
//    (attention_scalar_head, src/attention.c:606-642). Positions are split in chunks of kAttnChunk and merged with the
//    max-rescaling of split-K decoding (src/attention.c:700-802), so it agrees with the reference within fp32
//    rounding, not bitwise; each row's result depends only on its own position, so batched rows equal single rows.
//  - greedy sampling: the first maximum wins (sample_argmax, src/sampler.c:9-23)
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/kernels_cuda.h"
#include "common.cuh"
#include "kernels_cuda_internal.h"

namespace {

__global__ void embed_kernel(float *x, const int *tokens, const int8_t *q, const float *s, int rows, int dim, int gs,
                             int vocab) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)rows * dim)
    return;
  const int r = (int)(i / dim), c = (int)(i - (long long)r * dim);
  int tok = tokens[r];
  if (tok < 0 || tok >= vocab) {
    kc_raise(KC_ERR_BAD_ARGS);
    tok = 0;
  }
  const long long e = (long long)tok * dim + c;
  x[i] = __fmul_rn((float)q[e], s[e / gs]);
}

// Row r of q [rows][n_heads * hd] (stride q_ld) and k [rows][n_kv * hd] (stride kv_ld) rotated at position pos0 + r
// with the table [positions][2 * hd]; rotated k and v (stride kv_ld) stored into the caches [n_kv][seq][hd].
__global__ void rope_store_kernel(float *q, long long q_ld, const float *k, const float *v, long long kv_ld, float *kc,
                                  float *vc, const float *table, const int *pos_dev, int pos0, int rows, int n_heads,
                                  int n_kv, int hd, int seq) {
  const int half = hd / 2;
  const int per_row = (n_heads + n_kv) * half + n_kv * hd;  // rotations of q, k, then copies of v
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (long long)rows * per_row)
    return;
  const int r = (int)(id / per_row);
  int p = (int)(id - (long long)r * per_row);
  const int pos = (pos_dev ? *pos_dev : pos0) + r;
  if (pos < 0 || pos >= seq) {
    kc_raise(KC_ERR_BAD_ARGS);
    return;
  }
  if (p < (n_heads + n_kv) * half) {
    const float *t = table + (long long)pos * 2 * hd;
    const bool is_k = p >= n_heads * half;
    if (is_k)
      p -= n_heads * half;
    const int h = p / half, j = 2 * (p - h * half);
    const float *src = is_k ? k + r * kv_ld + h * hd + j : q + r * q_ld + h * hd + j;
    const float c = t[j], sn = t[hd + j + 1];
    const float a = src[0], b = src[1];
    const float o0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
    const float o1 = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
    float *dst = is_k ? kc + ((long long)h * seq + pos) * hd + j : q + r * q_ld + h * hd + j;
    dst[0] = o0, dst[1] = o1;
  } else {
    p -= (n_heads + n_kv) * half;
    const int h = p / hd, i = p - h * hd;
    vc[((long long)h * seq + pos) * hd + i] = v[r * kv_ld + h * hd + i];
  }
}

// Plain k_kv_store: count rows of n_kv * hd floats (stride src_ld) to positions pos0.. of the head-major cache.
__global__ void kv_store_kernel(float *cache, const float *src, long long src_ld, int pos0, int count, int n_kv, int hd,
                                int seq) {
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = n_kv * hd;
  if (id >= (long long)count * per_row)
    return;
  const int r = (int)(id / per_row), p = (int)(id - (long long)r * per_row);
  const int h = p / hd, i = p - h * hd;
  cache[((long long)h * seq + pos0 + r) * hd + i] = src[r * src_ld + p];
}

constexpr int kAttnThreads = 256;
constexpr int kAttnChunk = 128;  // positions per split
constexpr int kMaxGqa = 8;       // query heads per KV head handled by one CTA
constexpr int kMaxHd = 256;

// One CTA per (KV head g, split s, query row r): the kv_mul query heads of g against positions
// [s * chunk, min(pos + 1, (s + 1) * chunk)). Writes (max, sum, weighted V) partials; the last CTA of (g, r) to finish
// merges the splits and writes the output, quantized in gs-groups too when oq is set ((kv_mul * hd) % gs == 0).
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(
    float *out, long long out_ld, int8_t *oq, float *os, const float *q, long long q_ld, const float *kc,
    const float *vc, const int *pos_dev, int pos0, int n_kv, int kv_mul, int hd, int seq, int max_splits, float *part,
    int *counters, int gs) {
  __shared__ float qs[kMaxGqa * kMaxHd];
  __shared__ float sc[kMaxGqa][kAttnChunk];
  __shared__ float red[kMaxGqa][2];
  __shared__ int last;
  const int g = blockIdx.x, s = blockIdx.y, r = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = kAttnThreads / 32;
  const int pos = (pos_dev ? *pos_dev : pos0) + r;
  const int npos = pos + 1;
  const int nsplit = (npos + kAttnChunk - 1) / kAttnChunk;
  const int t0 = s * kAttnChunk, t1 = min(npos, t0 + kAttnChunk);
  const int nq = kv_mul;
  const float scale = sqrtf((float)hd);
  const long long stride = hd + 2;
  float *pbase = part + (((long long)r * n_kv + g) * max_splits) * nq * stride;
  if (s < nsplit && pos < seq) {
    for (int i = tid; i < nq * hd; i += kAttnThreads)
      qs[i] = q[r * q_ld + (long long)g * nq * hd + i];
    __syncthreads();
    const float *kh = kc + (long long)g * seq * hd;
    const float *vh = vc + (long long)g * seq * hd;
    // Scores: warp per position, lanes across head_dim.
    for (int t = t0 + warp; t < t1; t += nw) {
      const float *kt = kh + (long long)t * hd;
      float acc[kMaxGqa];
#pragma unroll
      for (int h = 0; h < kMaxGqa; h++)
        acc[h] = 0.0f;
      for (int i = lane; i < hd; i += 32) {
        const float kv = kt[i];
#pragma unroll
        for (int h = 0; h < kMaxGqa; h++)
          if (h < nq)
            acc[h] = fmaf(qs[h * hd + i], kv, acc[h]);
      }
#pragma unroll
      for (int h = 0; h < kMaxGqa; h++) {
        if (h >= nq)
          break;
        float d = acc[h];
#pragma unroll
        for (int o = 16; o; o >>= 1)
          d += __shfl_xor_sync(0xffffffffu, d, o);
        if (lane == 0)
          sc[h][t - t0] = d / scale;
      }
    }
    __syncthreads();
    // Chunk max and exp-sum per query head (warp h).
    if (warp < nq) {
      float m = -INFINITY;
      for (int t = lane; t < t1 - t0; t += 32)
        m = fmaxf(m, sc[warp][t]);
#pragma unroll
      for (int o = 16; o; o >>= 1)
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float l = 0.0f;
      for (int t = lane; t < t1 - t0; t += 32) {
        const float e = expf(sc[warp][t] - m);
        sc[warp][t] = e;
        l += e;
      }
#pragma unroll
      for (int o = 16; o; o >>= 1)
        l += __shfl_xor_sync(0xffffffffu, l, o);
      if (lane == 0)
        red[warp][0] = m, red[warp][1] = l;
    }
    __syncthreads();
    // Weighted values: thread per (head, dim), coalesced along dim.
    for (int i = tid; i < nq * hd; i += kAttnThreads) {
      const int h = i / hd, d = i - h * hd;
      float acc = 0.0f;
      for (int t = t0; t < t1; t++)
        acc = fmaf(sc[h][t - t0], vh[(long long)t * hd + d], acc);
      pbase[((long long)s * nq + h) * stride + 2 + d] = acc;
    }
    if (tid < nq) {
      pbase[((long long)s * nq + tid) * stride] = red[tid][0];
      pbase[((long long)s * nq + tid) * stride + 1] = red[tid][1];
    }
  } else if (pos >= seq && s == 0 && tid == 0) {
    kc_raise(KC_ERR_BAD_ARGS);
  }
  // The last CTA of (g, r) merges; every CTA of the grid's y extent counts in, including those past nsplit.
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int done = atomicAdd(&counters[r * n_kv + g], 1);
    last = done == (int)gridDim.y - 1;
  }
  __syncthreads();
  if (!last)
    return;
  __threadfence();
  if (tid == 0)
    counters[r * n_kv + g] = 0;  // ready for the next launch
  if (pos >= seq)
    return;
  __syncthreads();
  for (int i = tid; i < nq * hd; i += kAttnThreads) {
    const int h = i / hd, d = i - h * hd;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; sp++)
      M = fmaxf(M, __ldcg(pbase + ((long long)sp * nq + h) * stride));
    float L = 0.0f, O = 0.0f;
    for (int sp = 0; sp < nsplit; sp++) {
      const float *pp = pbase + ((long long)sp * nq + h) * stride;
      const float w = expf(__ldcg(pp) - M);
      L = fmaf(__ldcg(pp + 1), w, L);
      O = fmaf(__ldcg(pp + 2 + d), w, O);
    }
    qs[i] = O / L;
  }
  __syncthreads();
  float *orow = out + r * out_ld + (long long)g * nq * hd;
  for (int i = tid; i < nq * hd; i += kAttnThreads)
    orow[i] = qs[i];
  if (oq) {
    // Quantize this KV head's nq * hd outputs in gs-groups (k_quantize's rule), warp per group.
    const int groups = nq * hd / gs;
    int8_t *qrow = oq + r * out_ld + (long long)g * nq * hd;
    float *srow = os + r * (out_ld / gs) + (long long)g * nq * hd / gs;
    for (int grp = warp; grp < groups; grp += nw) {
      float mx = 0.0f;
      int bad = 0;
      for (int i = lane; i < gs; i += 32) {
        const float v = qs[grp * gs + i];
        bad |= !isfinite(v);
        mx = fmaxf(mx, fabsf(v));
      }
#pragma unroll
      for (int o = 16; o; o >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (__any_sync(0xffffffffu, bad) && lane == 0)
        kc_raise(KC_ERR_NONFINITE);
      const float scl = __fdiv_rn(mx, 127.0f);
      if (lane == 0)
        srow[grp] = scl;
      for (int i = lane; i < gs; i += 32)
        qrow[grp * gs + i] = (int8_t)quantize_value(qs[grp * gs + i], scl);
    }
  }
}

__global__ void add_kernel(float *x, const float *y, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n)
    x[i] = __fadd_rn(x[i], y[i]);
}

// 64-bit key whose unsigned maximum is the first maximum: order-preserving float bits, then the inverted index.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  unsigned b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (unsigned)(0xFFFFFFFFu - (unsigned)idx);
}

__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) { return a > b ? a : b; }

__global__ void argmax_kernel(unsigned long long *key, const float *logits, int n, int offset) {
  __shared__ unsigned long long best[32];
  unsigned long long k = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    k = umax64(k, argmax_key(logits[i], i + offset));
#pragma unroll
  for (int o = 16; o; o >>= 1)
    k = umax64(k, __shfl_xor_sync(0xffffffffu, k, o));
  if ((threadIdx.x & 31) == 0)
    best[threadIdx.x >> 5] = k;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++)
      k = umax64(k, best[w]);
    *key = umax64(best[0], k);
  }
}

// Greedy step bookkeeping on the device: token = index of *key; out[*step] = token; *token_in = token (the next
// step's input); *step += 1; *position += 1.
__global__ void greedy_advance_kernel(int *out, int *step, int *token_in, int *position, const unsigned long long *key) {
  const int idx = (int)(0xFFFFFFFFu - (unsigned)(*key & 0xFFFFFFFFull));
  if (out)
    out[*step] = idx;
  *token_in = idx;
  *step += 1;
  *position += 1;
}

// Seeded N(0, std) values by element index (SplitMix64 finalizer feeding Box-Muller), quantized to Q8 in gs-groups by
// k_quantize's rule: element (row, col) of tensor `tensor` is the same whatever shard holds it.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ float seeded_normal(uint64_t seed, uint64_t tensor, uint64_t index, float std) {
  const uint64_t h1 = mix64(seed ^ mix64(tensor * 0x9E3779B97F4A7C15ull + index));
  const uint64_t h2 = mix64(h1 + 0x632BE59BD9B4E019ull);
  const float u1 = ((float)(h1 >> 40) + 1.0f) * (1.0f / 16777217.0f);
  const float u2 = (float)(h2 >> 40) * (1.0f / 16777216.0f);
  return std * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__global__ void random_q8_kernel(int8_t *q, float *s, int rows, int cols, long long row0, long long col0,
                                 long long full_cols, unsigned long long seed, unsigned long long tensor, float std,
                                 int gs) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = cols / gs;
  const long long gid = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
  if (gid >= (long long)rows * groups)
    return;
  const int r = (int)(gid / groups), g = (int)(gid - (long long)r * groups);
  const long long base = (row0 + r) * full_cols + col0 + (long long)g * gs;
  float v[8];  // gs <= 256
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int i = lane + 32 * j;
    v[j] = i < gs ? seeded_normal(seed, tensor, (uint64_t)(base + i), std) : 0.0f;
    mx = fmaxf(mx, fabsf(v[j]));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1)
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float scl = __fdiv_rn(mx, 127.0f);
  if (lane == 0)
    s[(long long)r * groups + g] = scl;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int i = lane + 32 * j;
    if (i < gs)
      q[(long long)r * cols + (long long)g * gs + i] = (int8_t)quantize_value(v[j], scl);
  }
}

__global__ void fill_kernel(float *x, long long n, float v) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n)
    x[i] = v;
}

inline unsigned blocks_for(long long n, int t) { return (unsigned)((n + t - 1) / t); }

bool launched(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess)
    return true;
  return kc_fail("%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
}

int max_splits_for(int seq) { return (seq + kAttnChunk - 1) / kAttnChunk; }

bool attention_shape_ok(const char *name, const AttentionWork *w, int n_heads, int n_kv, int hd, int seq) {
  if (!w || !w->partial || !w->counters)
    return kc_fail("%s: attention work is not initialized", name);
  if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv || n_heads / n_kv > kMaxGqa || hd <= 0 || hd > kMaxHd || hd % 2)
    return kc_fail("%s: unsupported heads %d / KV heads %d / head_dim %d", name, n_heads, n_kv, hd);
  if (n_heads != w->n_heads || n_kv != w->n_kv_heads || hd != w->head_dim || seq != w->seq_len)
    return kc_fail("%s: shape differs from the one the work was initialized for", name);
  return true;
}

// Runs `rows` query rows in waves of the work's row capacity. With device positions (graph replay) the grid covers
// every split of the context and all rows go in one wave.
bool attention_rows(const char *name, float *out, long long out_ld, int8_t *oq, float *os, const float *q,
                    long long q_ld, const float *kc, const float *vc, AttentionWork *w, int n_heads, int n_kv, int hd,
                    int seq, const int *pos_dev, int pos0, int rows, int gs) {
  if (!attention_shape_ok(name, w, n_heads, n_kv, hd, seq))
    return false;
  if (oq && (gs <= 0 || (n_heads / n_kv * hd) % gs || out_ld % gs))
    return kc_fail("%s: group size %d does not divide a KV head's outputs", name, gs);
  if (!pos_dev && (pos0 < 0 || pos0 + rows > seq))
    return kc_fail("%s: positions %d..%d outside the context of %d", name, pos0, pos0 + rows - 1, seq);
  if (pos_dev && rows > w->rows)
    return kc_fail("%s: device positions need all %d rows in one wave (work holds %d)", name, rows, w->rows);
  const int max_splits = max_splits_for(seq);
  for (int r0 = 0; r0 < rows; r0 += w->rows) {
    const int n = rows - r0 < w->rows ? rows - r0 : w->rows;
    const int splits = pos_dev ? max_splits : max_splits_for(pos0 + r0 + n);
    dim3 grid(n_kv, splits, n);
    attention_kernel<<<grid, kAttnThreads, 0, kc_stream()>>>(
        out + r0 * out_ld, out_ld, oq ? oq + r0 * out_ld : nullptr, oq ? os + r0 * (out_ld / gs) : nullptr,
        q + r0 * q_ld, q_ld, kc, vc, pos_dev, pos0 + r0, n_kv, n_heads / n_kv, hd, seq, max_splits, w->partial,
        w->counters, gs);
    if (!launched(name))
      return false;
  }
  return true;
}

}  // namespace

extern "C" {

// ---- K/V cache (head-major) ---------------------------------------------------------------------------------------

void k_kv_strides(int n_kv_heads, int head_dim, int seq_len, size_t *pos_stride, size_t *head_base) {
  (void)n_kv_heads;
  *pos_stride = (size_t)head_dim;
  *head_base = (size_t)seq_len * head_dim;
}

void k_kv_store(float *cache, const float *src, size_t src_ld, int pos0, int count, int n_kv_heads, int head_dim,
                int seq_len) {
  if (count < 0 || pos0 < 0 || pos0 + count > seq_len || n_kv_heads <= 0 || head_dim <= 0 ||
      src_ld < (size_t)n_kv_heads * head_dim) {
    kc_fail("k_kv_store: invalid shape pos0=%d count=%d seq_len=%d", pos0, count, seq_len);
    return;
  }
  const long long total = (long long)count * n_kv_heads * head_dim;
  if (!total)
    return;
  kv_store_kernel<<<blocks_for(total, 256), 256, 0, kc_stream()>>>(cache, src, (long long)src_ld, pos0, count,
                                                                   n_kv_heads, head_dim, seq_len);
  launched("k_kv_store");
}

void k_rope_kv_store_rows(float *q, size_t q_ld, const float *k, const float *v, size_t kv_ld, float *key_cache,
                          float *value_cache, const float *table, const int *position, int pos0, int rows, int n_heads,
                          int n_kv_heads, int head_dim, int seq_len) {
  if (rows < 0 || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || head_dim % 2 ||
      q_ld < (size_t)n_heads * head_dim || kv_ld < (size_t)n_kv_heads * head_dim ||
      (!position && (pos0 < 0 || pos0 + rows > seq_len))) {
    kc_fail("k_rope_kv_store_rows: invalid shape");
    return;
  }
  const long long total = (long long)rows * ((n_heads + n_kv_heads) * (head_dim / 2) + n_kv_heads * head_dim);
  if (!total)
    return;
  rope_store_kernel<<<blocks_for(total, 256), 256, 0, kc_stream()>>>(q, (long long)q_ld, k, v, (long long)kv_ld,
                                                                      key_cache, value_cache, table, position, pos0,
                                                                      rows, n_heads, n_kv_heads, head_dim, seq_len);
  launched("k_rope_kv_store_rows");
}

// ---- attention ----------------------------------------------------------------------------------------------------

size_t k_attention_bytes_rows(int n_heads, int n_kv_heads, int head_dim, int seq_len, int rows) {
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || seq_len <= 0 || rows <= 0)
    return 0;
  const size_t partial = (size_t)rows * n_heads * max_splits_for(seq_len) * (head_dim + 2) * sizeof(float);
  const size_t counters = (size_t)rows * n_kv_heads * sizeof(int);
  return ((partial + 255) & ~(size_t)255) + counters;
}

void k_attention_init_rows(AttentionWork *work, int n_heads, int n_kv_heads, int head_dim, int seq_len, int rows,
                           void *memory) {
  const size_t bytes = k_attention_bytes_rows(n_heads, n_kv_heads, head_dim, seq_len, rows);
  memset(work, 0, sizeof(*work));
  if (!bytes) {
    kc_fail("k_attention_init_rows: invalid shape");
    return;
  }
  char *base = static_cast<char *>(memory);
  int external = 1;
  if (!base) {
    if (cudaMalloc(&base, bytes) != cudaSuccess) {
      cudaGetLastError();
      kc_fail("k_attention_init_rows: cannot allocate %zu bytes of attention work", bytes);
      return;
    }
    external = 0;
  }
  const size_t partial = (size_t)rows * n_heads * max_splits_for(seq_len) * (head_dim + 2) * sizeof(float);
  const size_t counters_at = (partial + 255) & ~(size_t)255;
  if (cudaMemsetAsync(base + counters_at, 0, (size_t)rows * n_kv_heads * sizeof(int), kc_stream()) != cudaSuccess) {
    cudaGetLastError();
    kc_fail("k_attention_init_rows: cannot clear the merge counters");
  }
  work->partial = reinterpret_cast<float *>(base);
  work->counters = reinterpret_cast<int *>(base + counters_at);
  work->max_chunks = max_splits_for(seq_len);
  work->n_heads = n_heads;
  work->n_kv_heads = n_kv_heads;
  work->head_dim = head_dim;
  work->seq_len = seq_len;
  work->rows = rows;
  work->external = external;
  work->capacity = partial / sizeof(float);
}

void k_attention_free(AttentionWork *work) {
  if (work->partial && !work->external)
    cudaFree(work->partial);
  memset(work, 0, sizeof(*work));
}

void k_attention_kv(float *out, const float *q, const float *key_cache, const float *value_cache, float *att,
                    AttentionWork *work, int n_heads, int n_kv_heads, int head_dim, int seq_len, int position) {
  (void)att;
  const long long ld = (long long)n_heads * head_dim;
  attention_rows("k_attention_kv", out, ld, nullptr, nullptr, q, ld, key_cache, value_cache, work, n_heads,
                 n_kv_heads, head_dim, seq_len, nullptr, position, 1, 0);
}

void k_attention_batch_kv(float *out, const float *q, const float *key_cache, const float *value_cache, float *att,
                          AttentionWork *work, int n_heads, int n_kv_heads, int head_dim, int seq_len, int pos0,
                          int m) {
  (void)att;
  const long long ld = (long long)n_heads * head_dim;
  attention_rows("k_attention_batch_kv", out, ld, nullptr, nullptr, q, ld, key_cache, value_cache, work, n_heads,
                 n_kv_heads, head_dim, seq_len, nullptr, pos0, m, 0);
}

void k_attention_q8_rows(float *out, int8_t *oq, float *os, const float *q, const float *key_cache,
                         const float *value_cache, AttentionWork *work, int n_heads, int n_kv_heads, int head_dim,
                         int seq_len, const int *position, int pos0, int rows, int gs) {
  const long long ld = (long long)n_heads * head_dim;
  attention_rows("k_attention_q8_rows", out, ld, oq, os, q, ld, key_cache, value_cache, work, n_heads, n_kv_heads,
                 head_dim, seq_len, position, pos0, rows, gs);
}

// ---- embedding, residual, sampling --------------------------------------------------------------------------------

void k_embed_q8_rows(float *x, const int *tokens, K8Weight embed, int rows, int dim, int gs, int vocab) {
  if (rows < 0 || dim <= 0 || gs <= 0 || dim % gs || vocab <= 0 || !embed.q || !embed.s) {
    kc_fail("k_embed_q8_rows: invalid arguments");
    return;
  }
  if (!rows)
    return;
  embed_kernel<<<blocks_for((long long)rows * dim, 256), 256, 0, kc_stream()>>>(x, tokens, embed.q, embed.s, rows,
                                                                                 dim, gs, vocab);
  launched("k_embed_q8_rows");
}

void k_add(float *x, const float *y, size_t n) {
  if (!n)
    return;
  add_kernel<<<blocks_for((long long)n, 256), 256, 0, kc_stream()>>>(x, y, (long long)n);
  launched("k_add");
}

void k_argmax_key(unsigned long long *key, const float *logits, int n, int offset) {
  if (n <= 0) {
    kc_fail("k_argmax_key: empty logits");
    return;
  }
  argmax_kernel<<<1, 1024, 0, kc_stream()>>>(key, logits, n, offset);
  launched("k_argmax_key");
}

void k_greedy_advance(int *out, int *step, int *token, int *position, const unsigned long long *key) {
  greedy_advance_kernel<<<1, 1, 0, kc_stream()>>>(out, step, token, position, key);
  launched("k_greedy_advance");
}

// ---- seeded benchmark weights -------------------------------------------------------------------------------------

void k_random_q8(int8_t *q, float *s, int rows, int cols, size_t row0, size_t col0, size_t full_cols,
                 unsigned long long seed, unsigned long long tensor, float std, int gs) {
  if (rows < 0 || cols <= 0 || gs < 32 || gs > 256 || gs % 32 || cols % gs || col0 % gs ||
      col0 + cols > full_cols) {
    kc_fail("k_random_q8: invalid shape rows=%d cols=%d gs=%d", rows, cols, gs);
    return;
  }
  const long long warps = (long long)rows * (cols / gs);
  if (!warps)
    return;
  random_q8_kernel<<<blocks_for(warps, 8), 256, 0, kc_stream()>>>(q, s, rows, cols, (long long)row0, (long long)col0,
                                                                   (long long)full_cols, seed, tensor, std, gs);
  launched("k_random_q8");
}

void k_fill(float *x, size_t n, float value) {
  if (!n)
    return;
  fill_kernel<<<blocks_for((long long)n, 256), 256, 0, kc_stream()>>>(x, (long long)n, value);
  launched("k_fill");
}

}  // extern "C"
