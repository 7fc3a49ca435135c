// Per-token kernels of the GPU forward pass (the C11 engine, engine.c): embedding dequantization, RoPE fused with the
// K/V store, residual add, greedy argmax, and the seeded Q8 generator of the benchmark models (attention is in
// attention.cu).
//
// Reference semantics (LucianCrainic/llama3.x.c):
//  - embedding: x[i] = (float)q[row * dim + i] * s[(row * dim + i) / gs]                  (src/tp.c:395-396)
//  - RoPE from the host-built table (k_rope_table / k_rope_apply, src/kernels_simd.c:194-227), bitwise
//  - K/V cache head-major [kv_head][position][head_dim] (k_kv_store / k_kv_strides, src/attention.c:1415-1432)
//  - attention: attention.cu, bitwise the reference's split (one row) and tiled (batch) variants
//  - greedy sampling: the first maximum wins (sample_argmax, src/sampler.c:9-23)
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/kernels_cuda.h"
#include "common.cuh"
#include "kernels_cuda_internal.h"

namespace {

__global__ void embed_kernel(float *x, const int *tokens, const int8_t *q, const float *s, int rows, int dim, int gs,
                             int vocab) {
  pdl_wait();
  pdl_launch_dependents();
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
  pdl_wait();
  pdl_launch_dependents();
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
  pdl_wait();
  pdl_launch_dependents();
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = n_kv * hd;
  if (id >= (long long)count * per_row)
    return;
  const int r = (int)(id / per_row), p = (int)(id - (long long)r * per_row);
  const int h = p / hd, i = p - h * hd;
  cache[((long long)h * seq + pos0 + r) * hd + i] = src[r * src_ld + p];
}

__global__ void add_kernel(float *x, const float *y, long long n) {
  pdl_wait();
  pdl_launch_dependents();
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

__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) {
  return a > b ? a : b;
}

// Each CTA reduces its share of the logits to one key and folds it into *key with a 64-bit atomic maximum (the
// caller leaves *key at 0 beforehand: a fresh buffer, or k_greedy_advance's reset).
__global__ void argmax_kernel(unsigned long long *key, const float *logits, int n, int offset) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ unsigned long long best[32];
  unsigned long long k = 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
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
    atomicMax(key, umax64(best[0], k));
  }
}

// Greedy step bookkeeping on the device: token = index of *key; out[*step] = token; *token_in = token (the next
// step's input); *step += 1; *position += 1; *key = 0 for the next argmax.
__global__ void greedy_advance_kernel(int *out, int *step, int *token_in, int *position, unsigned long long *key) {
  pdl_wait();
  pdl_launch_dependents();
  const int idx = (int)(0xFFFFFFFFu - (unsigned)(*key & 0xFFFFFFFFull));
  *key = 0;
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
  pdl_wait();
  pdl_launch_dependents();
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
  pdl_wait();
  pdl_launch_dependents();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n)
    x[i] = v;
}

inline unsigned blocks_for(long long n, int t) { return (unsigned)((n + t - 1) / t); }

bool launched(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    kc_count_launch();
    return true;
  }
  return kc_fail("%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
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
  kc_launch_pdl(kv_store_kernel, blocks_for(total, 256), 256, 0, kc_stream(), cache, src, (long long)src_ld, pos0,
      count, n_kv_heads, head_dim, seq_len);
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
  kc_launch_pdl(rope_store_kernel, blocks_for(total, 256), 256, 0, kc_stream(), q, (long long)q_ld, k, v,
      (long long)kv_ld, key_cache, value_cache, table, position, pos0, rows, n_heads, n_kv_heads, head_dim, seq_len);
  launched("k_rope_kv_store_rows");
}

// ---- embedding, residual, sampling --------------------------------------------------------------------------------

void k_embed_q8_rows(float *x, const int *tokens, K8Weight embed, int rows, int dim, int gs, int vocab) {
  if (rows < 0 || dim <= 0 || gs <= 0 || dim % gs || vocab <= 0 || !embed.q || !embed.s) {
    kc_fail("k_embed_q8_rows: invalid arguments");
    return;
  }
  if (!rows)
    return;
  kc_launch_pdl(embed_kernel, blocks_for((long long)rows * dim, 256), 256, 0, kc_stream(), x, tokens, embed.q, embed.s,
      rows, dim, gs, vocab);
  launched("k_embed_q8_rows");
}

void k_add(float *x, const float *y, size_t n) {
  if (!n)
    return;
  kc_launch_pdl(add_kernel, blocks_for((long long)n, 256), 256, 0, kc_stream(), x, y, (long long)n);
  launched("k_add");
}

void k_argmax_key(unsigned long long *key, const float *logits, int n, int offset) {
  if (n <= 0) {
    kc_fail("k_argmax_key: empty logits");
    return;
  }
  const int blocks = (n + 4 * 256 - 1) / (4 * 256);
  kc_launch_pdl(argmax_kernel, blocks < 2 * kc_device_sms() ? blocks : 2 * kc_device_sms(), 256, 0, kc_stream(), key,
      logits, n, offset);
  launched("k_argmax_key");
}

void k_greedy_advance(int *out, int *step, int *token, int *position, unsigned long long *key) {
  kc_launch_pdl(greedy_advance_kernel, 1, 1, 0, kc_stream(), out, step, token, position, key);
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
  kc_launch_pdl(random_q8_kernel, blocks_for(warps, 8), 256, 0, kc_stream(), q, s, rows, cols, (long long)row0,
      (long long)col0, (long long)full_cols, seed, tensor, std, gs);
  launched("k_random_q8");
}

void k_fill(float *x, size_t n, float value) {
  if (!n)
    return;
  kc_launch_pdl(fill_kernel, blocks_for((long long)n, 256), 256, 0, kc_stream(), x, (long long)n, value);
  launched("k_fill");
}

}  // extern "C"
