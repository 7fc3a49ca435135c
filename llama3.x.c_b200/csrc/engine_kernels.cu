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

constexpr int kAttnThreads = 256;
constexpr int kAttnChunk = 64;     // positions per split: split c covers [64 c, 64 c + 64), whatever the row
constexpr int kMaxGqa = 8;         // query heads per KV head
constexpr int kMaxHd = 128;
constexpr int kDecodeStages = 1;   // K/V chunk buffers of a decode CTA: one, so two CTAs fit per SM

// Dynamic shared memory of the attention kernels: `stages` buffers of one chunk's K and V rows (filled by bulk copies),
// the row's query heads, the chunk's scores, the position-group partial sums of P.V, per-head (max, sum) and one copy
// barrier per stage.
struct AttnSmem {
  float *K[2], *V[2];  // stage buffers (both entries alias stage 0 when there is one stage)
  float *qs, *sc, *pv, *red;
  uint64_t *bar;
};

__host__ __device__ inline size_t attn_smem_bytes(int hd, int stages) {
  return ((size_t)stages * 2 * kAttnChunk * hd + kMaxGqa * kMaxHd + kMaxGqa * kAttnChunk + kAttnThreads * kMaxGqa +
          2 * kMaxGqa) * sizeof(float) + kDecodeStages * sizeof(uint64_t);
}

__device__ inline AttnSmem attn_smem(int hd, int stages) {
  extern __shared__ __align__(16) float attn_dyn[];
  AttnSmem m;
  float *p = attn_dyn;
  for (int i = 0; i < 2; i++) {
    m.K[i] = p;
    m.V[i] = p + kAttnChunk * hd;
    if (i + 1 < stages)
      p += 2 * kAttnChunk * hd;
  }
  p += 2 * kAttnChunk * hd;
  m.qs = p;
  m.sc = m.qs + kMaxGqa * kMaxHd;
  m.pv = m.sc + kMaxGqa * kAttnChunk;
  m.red = m.pv + kAttnThreads * kMaxGqa;
  m.bar = reinterpret_cast<uint64_t *>(m.red + 2 * kMaxGqa);  // every size above is a multiple of 2 floats
  return m;
}

// Thread 0 issues the bulk copies of rows [t0, t0 + n) of KV head g's K and V (contiguous in the head-major cache)
// into stage `st`, completing on that stage's barrier.
__device__ inline void issue_chunk(const AttnSmem &m, int st, const float *kc, const float *vc, int g, int seq, int hd,
                                   int t0, int n) {
  const unsigned bytes = (unsigned)n * hd * sizeof(float);
  mbar_arrive_expect_tx(m.bar + st, 2 * bytes);
  bulk_g2s(st ? m.K[1] : m.K[0], kc + ((long long)g * seq + t0) * hd, bytes, m.bar + st);
  bulk_g2s(st ? m.V[1] : m.V[0], vc + ((long long)g * seq + t0) * hd, bytes, m.bar + st);
}

// Bounded wait for a stage, with the same outcome in every thread of the CTA.
__device__ inline bool wait_chunk(const AttnSmem &m, int st, unsigned parity) {
  return __syncthreads_and(mbar_wait_bounded(m.bar + st, parity));
}

// One row's partial over the first n_t positions of the chunk in K/V: per query head h of the KV head,
// pdst[h] = (max score, sum of exp(score - max), sum of exp(score - max) v). The arithmetic order depends only on
// (n_t, nq, hd) and the position within the chunk; decode and prefill both come through here, so a row's result does
// not depend on which kernel ran it.
__device__ inline void chunk_partial(const AttnSmem &m, const float *K, const float *V, const float *qg, int n_t,
                                     int nq, int hd, float *pdst) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float scale = sqrtf((float)hd);
  const int stride = hd + 2, hd4 = hd / 4;
  for (int i = tid; i < nq * hd; i += kAttnThreads)
    m.qs[i] = qg[i];
  __syncthreads();
  // Scores: a thread per (head, position); the float4 index is rotated by the position so the 32 lanes of a warp hit
  // 32 different banks, and four partial sums give the FMA chain independent links.
  for (int pair = tid; pair < nq * kAttnChunk; pair += kAttnThreads) {
    const int h = pair / kAttnChunk, p = pair - h * kAttnChunk;
    if (p < n_t) {
      const float4 *k4 = reinterpret_cast<const float4 *>(K + p * hd);
      const float4 *q4 = reinterpret_cast<const float4 *>(m.qs + h * hd);
      float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
      int j = p % hd4;
#pragma unroll 4
      for (int i = 0; i < hd4; i++) {
        const float4 kv = k4[j], qv = q4[j];
        a0 = fmaf(qv.x, kv.x, a0);
        a1 = fmaf(qv.y, kv.y, a1);
        a2 = fmaf(qv.z, kv.z, a2);
        a3 = fmaf(qv.w, kv.w, a3);
        j = j + 1 == hd4 ? 0 : j + 1;
      }
      m.sc[h * kAttnChunk + p] = ((a0 + a1) + (a2 + a3)) / scale;
    }
  }
  __syncthreads();
  // Chunk max and exp-sum per head (warp per head, two positions per lane).
  for (int h = warp; h < nq; h += kAttnThreads / 32) {
    float *sch = m.sc + h * kAttnChunk;
    const float s0 = lane < n_t ? sch[lane] : -INFINITY, s1 = lane + 32 < n_t ? sch[lane + 32] : -INFINITY;
    float mx = fmaxf(s0, s1);
#pragma unroll
    for (int o = 16; o; o >>= 1)
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float e0 = lane < n_t ? expf(s0 - mx) : 0.0f, e1 = lane + 32 < n_t ? expf(s1 - mx) : 0.0f;
    if (lane < n_t)
      sch[lane] = e0;
    if (lane + 32 < n_t)
      sch[lane + 32] = e1;
    float l = e0 + e1;
#pragma unroll
    for (int o = 16; o; o >>= 1)
      l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0)
      m.red[2 * h] = mx, m.red[2 * h + 1] = l;
  }
  __syncthreads();
  // Weighted values: a thread per (position group, dim) accumulates every head of its dim over its group's positions
  // (nq independent chains); the groups' sums are added in group order.
  const int groups = kAttnThreads / hd, grp = tid / hd, d = tid - grp * hd;
  if (grp < groups) {
    const int per = (n_t + groups - 1) / groups, t0 = grp * per, t1 = min(n_t, t0 + per);
    float acc[kMaxGqa];
#pragma unroll
    for (int h = 0; h < kMaxGqa; h++)
      acc[h] = 0.0f;
    for (int t = t0; t < t1; t++) {
      const float v = V[t * hd + d];
#pragma unroll
      for (int h = 0; h < kMaxGqa; h++)
        if (h < nq)
          acc[h] = fmaf(m.sc[h * kAttnChunk + t], v, acc[h]);
    }
#pragma unroll
    for (int h = 0; h < kMaxGqa; h++)
      if (h < nq)
        m.pv[(grp * kMaxGqa + h) * hd + d] = acc[h];
  }
  __syncthreads();
  for (int i = tid; i < nq * hd; i += kAttnThreads) {
    const int h = i / hd, dd = i - h * hd;
    float sum = m.pv[h * hd + dd];
    for (int g2 = 1; g2 < groups; g2++)
      sum += m.pv[(g2 * kMaxGqa + h) * hd + dd];
    pdst[h * stride + 2 + dd] = sum;
  }
  if (tid < nq) {
    pdst[tid * stride] = m.red[2 * tid];
    pdst[tid * stride + 1] = m.red[2 * tid + 1];
  }
  __syncthreads();  // qs, sc, pv and red are reused next
}

// Decode: gridDim.y CTAs per (KV head g, row r); CTA y takes chunks y, y + gridDim.y, ... and writes each chunk's
// partial; attention_combine_kernel merges them.
__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(
    const float *q, long long q_ld, const float *kc, const float *vc, const int *pos_dev, int pos0, int n_kv, int nq,
    int hd, int seq, int max_splits, float *part) {
  pdl_wait();
  pdl_launch_dependents();
  const AttnSmem m = attn_smem(hd, kDecodeStages);
  const int g = blockIdx.x, y = blockIdx.y, r = blockIdx.z, tid = threadIdx.x, step = gridDim.y;
  const int pos = (pos_dev ? *pos_dev : pos0) + r;
  const bool valid = pos >= 0 && pos < seq;
  const int npos = pos + 1, nsplit = (npos + kAttnChunk - 1) / kAttnChunk;
  const int stride = hd + 2;
  float *pbase = part + ((long long)r * n_kv + g) * max_splits * nq * stride;
  if (tid == 0) {
    for (int i = 0; i < kDecodeStages; i++)
      mbar_init(m.bar + i, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (!valid) {
    if (y == 0 && tid == 0)
      kc_raise(KC_ERR_BAD_ARGS);
  } else if (y < nsplit) {
    const float *qg = q + r * q_ld + (long long)g * nq * hd;
    if (tid == 0)
      issue_chunk(m, 0, kc, vc, g, seq, hd, y * kAttnChunk, min(npos - y * kAttnChunk, kAttnChunk));
    int k = 0, issued = 1;
    for (int c = y; c < nsplit; c += step, k++) {
      const int st = k % kDecodeStages, next = c + step;
      const bool more = next < nsplit;
      if (kDecodeStages > 1 && more && tid == 0)  // the other stage's chunk is done: load the next one meanwhile
        issue_chunk(m, (k + 1) % kDecodeStages, kc, vc, g, seq, hd, next * kAttnChunk,
                    min(npos - next * kAttnChunk, kAttnChunk));
      issued += kDecodeStages > 1 && more;
      if (!wait_chunk(m, st, (k / kDecodeStages) & 1)) {
        for (int j = k; j < issued; j++)  // let every copy in flight land (bounded) before leaving
          mbar_wait_bounded(m.bar + j % kDecodeStages, (j / kDecodeStages) & 1);
        break;
      }
      chunk_partial(m, st ? m.K[1] : m.K[0], st ? m.V[1] : m.V[0], qg, min(npos - c * kAttnChunk, kAttnChunk), nq,
                    hd, pbase + (long long)c * nq * stride);
      if (kDecodeStages == 1 && more && tid == 0)  // one stage: its buffer is free once the math above is done
        issue_chunk(m, 0, kc, vc, g, seq, hd, next * kAttnChunk, min(npos - next * kAttnChunk, kAttnChunk));
      issued += kDecodeStages == 1 && more;
    }
  }
}

// ---- prefill: flash-style, register-tiled fp32 -------------------------------------------------------------------
// One CTA per (KV head g, block of kFlashQ query vectors = kFlashQ / nq rows x the nq query heads of g). It streams
// the 64-position K/V chunks of the block's causal range through shared memory (one bulk copy per tensor and chunk)
// and keeps an online softmax per query: S = Q K^T / sqrt(hd) on 4 x 4 register tiles (queries x positions, the k walk
// rotated by the tile's position block so the lanes of a warp spread over the banks), then running max / sum, then
// O = O * exp(m_old - m_new) + P V on 4 x (hd / 16) tiles. No split partials, no merge. The summation order differs
// from the decode kernel's, so a batched row agrees with the same position decoded alone within fp32 rounding.
constexpr int kFlashQ = 64;      // query vectors per CTA
constexpr int kFlashChunk = 64;  // positions per K/V chunk

// The K chunk's region also holds P ([kFlashQ][kFlashChunk]) once the scores no longer need K: it is the larger of
// the two.
__host__ __device__ constexpr int flash_kp_floats(int hd) {
  return kFlashChunk * hd > kFlashQ * kFlashChunk ? kFlashChunk * hd : kFlashQ * kFlashChunk;
}

__host__ __device__ inline size_t flash_smem_bytes(int hd) {
  // K / P, the V chunk, the Q tile, per-query max / sum / correction, the barrier.
  return ((size_t)flash_kp_floats(hd) + 2 * kFlashChunk * hd + 3 * kFlashQ) * sizeof(float) + 16;
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads, 2) attention_flash_kernel(
    float *out, long long out_ld, const float *q, long long q_ld, const float *kc, const float *vc,
    const int *pos_dev, int pos0, int rows, int n_kv, int nq, int seq) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) float fl[];
  float *K = fl, *V = K + flash_kp_floats(HD), *Q = V + kFlashChunk * HD;
  float *P = K;  // [kFlashQ][kFlashChunk], written after the scores no longer need K
  float *rowm = Q + kFlashQ * HD, *rowl = rowm + kFlashQ, *corr = rowl + kFlashQ;
  uint64_t *bar = reinterpret_cast<uint64_t *>(corr + kFlashQ);
  constexpr int DB = HD / 16;  // output dims per thread
  const int g = blockIdx.x, tid = threadIdx.x, R = kFlashQ / nq;
  const int r0 = blockIdx.y * R, r1 = min(rows, r0 + R), nv = (r1 - r0) * nq;
  const int base = pos_dev ? *pos_dev : pos0;
  const int last_pos = min(base + r1 - 1, seq - 1);
  if (base + r0 < 0 || base + r0 >= seq) {
    if (tid == 0)
      kc_raise(KC_ERR_BAD_ARGS);
    return;
  }
  // Query v = (row - r0) * nq + h: a row's nq heads are contiguous. 16-byte loads, 8 in flight per thread.
  {
    constexpr int per4 = kFlashQ * HD / 4, B = 8;
    for (int base = tid; base < per4; base += kAttnThreads * B) {
      float4 r[B];
#pragma unroll
      for (int b = 0; b < B; b++) {
        const int i = base + b * kAttnThreads, v = i / (HD / 4), d4 = i - v * (HD / 4);
        r[b] = i < per4 && v < nv ? reinterpret_cast<const float4 *>(q + (r0 + v / nq) * q_ld +
                                                                      (long long)(g * nq + v % nq) * HD)[d4]
                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (int b = 0; b < B; b++)
        if (base + b * kAttnThreads < per4)
          reinterpret_cast<float4 *>(Q)[base + b * kAttnThreads] = r[b];
    }
  }
  if (tid < kFlashQ)
    rowm[tid] = -INFINITY, rowl[tid] = 0.0f;
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const float scale = sqrtf((float)HD);
  const int qi = tid >> 4, pi = tid & 15;  // S tile: queries 4 qi.., positions 4 pi..; O tile: queries 4 qi.., dims DB pi..
  float o[4][DB];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int d = 0; d < DB; d++)
      o[i][d] = 0.0f;
  const int nchunks = last_pos / kFlashChunk + 1;
  for (int c = 0; c < nchunks; c++) {
    const int t0 = c * kFlashChunk, n = min(kFlashChunk, last_pos + 1 - t0);
    if (tid == 0) {
      const unsigned bytes = (unsigned)n * HD * sizeof(float);
      mbar_arrive_expect_tx(bar, 2 * bytes);
      bulk_g2s(K, kc + ((long long)g * seq + t0) * HD, bytes, bar);
      bulk_g2s(V, vc + ((long long)g * seq + t0) * HD, bytes, bar);
    }
    if (!__syncthreads_and(mbar_wait_bounded(bar, c & 1))) {
      mbar_wait_bounded(bar, c & 1);  // let the copies land (bounded) before leaving
      return;
    }
    float sc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++)
        sc[i][j] = 0.0f;
#pragma unroll 2
    for (int kk = 0; kk < HD / 4; kk++) {
      const int k4 = (kk + pi) & (HD / 4 - 1);
      float4 kv[4], qv[4];
#pragma unroll
      for (int j = 0; j < 4; j++)
        kv[j] = reinterpret_cast<const float4 *>(K + (4 * pi + j) * HD)[k4];
#pragma unroll
      for (int i = 0; i < 4; i++)
        qv[i] = reinterpret_cast<const float4 *>(Q + (4 * qi + i) * HD)[k4];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
          sc[i][j] = fmaf(qv[i].x, kv[j].x, sc[i][j]);
          sc[i][j] = fmaf(qv[i].y, kv[j].y, sc[i][j]);
          sc[i][j] = fmaf(qv[i].z, kv[j].z, sc[i][j]);
          sc[i][j] = fmaf(qv[i].w, kv[j].w, sc[i][j]);
        }
    }
    __syncthreads();  // K is overwritten by P below
    float cf[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int v = 4 * qi + i;
      const int pos = base + r0 + v / nq;  // the query's own position: it attends to t <= pos
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int p = 4 * pi + j;
        sc[i][j] = (v < nv && p < n && t0 + p <= pos) ? sc[i][j] / scale : -INFINITY;
        mx = fmaxf(mx, sc[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = rowm[v], m_new = fmaxf(m_old, mx);
      cf[i] = m_new == -INFINITY ? 1.0f : expf(m_old - m_new);
      float sum = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float e = sc[i][j] == -INFINITY ? 0.0f : expf(sc[i][j] - m_new);
        P[v * kFlashChunk + 4 * pi + j] = e;
        sum += e;
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1)
        sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (pi == 0) {
        rowm[v] = m_new;
        rowl[v] = fmaf(rowl[v], cf[i], sum);
      }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int d = 0; d < DB; d++)
        o[i][d] *= cf[i];
    for (int p = 0; p < n; p++) {
      float pv[4], vv[DB];
#pragma unroll
      for (int i = 0; i < 4; i++)
        pv[i] = P[(4 * qi + i) * kFlashChunk + p];
#pragma unroll
      for (int d = 0; d < DB; d++)
        vv[d] = V[p * HD + pi * DB + d];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int d = 0; d < DB; d++)
          o[i][d] = fmaf(pv[i], vv[d], o[i][d]);
    }
    __syncthreads();  // K/P and V are refilled by the next chunk
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int v = 4 * qi + i;
    if (v >= nv)
      continue;
    const float inv = rowl[v];
    float *dst = out + (r0 + v / nq) * out_ld + (long long)(g * nq + v % nq) * HD + pi * DB;
#pragma unroll
    for (int d = 0; d < DB; d++)
      dst[d] = o[i][d] / inv;
  }
}

constexpr int kCombineGroups = kAttnThreads / 32;  // split groups, a warp each
constexpr int kCombineDims = 64;                    // outputs per CTA (at most): two per lane

// Merges a row's chunk partials for one query head and a block of min(hd, 64) dims: one CTA per (head, dim block,
// row). The splits are cut into kCombineGroups contiguous groups of ceil(nsplit / kCombineGroups); warp k sums its
// group in split order (weights exp(max_s - max)), then the groups are added in group order, so the result depends
// only on the partials, never on which kernel wrote them. With oq set and a block of exactly gs dims, the block is
// also quantized (k_quantize's rule) as one group.
__global__ void __launch_bounds__(kAttnThreads) attention_combine_kernel(
    float *out, long long out_ld, int8_t *oq, float *os, const int *pos_dev, int pos0, int n_kv, int nq, int hd,
    int seq, int max_splits, const float *part, int gs) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float po[kCombineGroups][kCombineDims], pl[kCombineGroups], red[kCombineGroups], vo[kCombineDims];
  const int dims = hd < kCombineDims ? hd : kCombineDims, blocks = hd / dims;
  const int h = blockIdx.x / blocks, d0 = (blockIdx.x - h * blocks) * dims, r = blockIdx.y;
  const int g = h / nq, hh = h - g * nq, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pos = (pos_dev ? *pos_dev : pos0) + r;
  if (pos < 0 || pos >= seq) {
    if (blockIdx.x == 0 && tid == 0)
      kc_raise(KC_ERR_BAD_ARGS);
    return;
  }
  const int stride = hd + 2, nsplit = (pos + kAttnChunk) / kAttnChunk;
  const long long sstep = (long long)nq * stride;  // from split s to split s + 1
  const float *pb = part + (((long long)r * n_kv + g) * max_splits * nq + hh) * stride;
  // The maximum over the splits (order-independent).
  float mx = -INFINITY;
  for (int s = tid; s < nsplit; s += kAttnThreads)
    mx = fmaxf(mx, __ldcg(pb + s * sstep));
#pragma unroll
  for (int o = 16; o; o >>= 1)
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0)
    red[warp] = mx;
  __syncthreads();
  float M = red[0];
  for (int k = 1; k < kCombineGroups; k++)
    M = fmaxf(M, red[k]);
  // Warp k: its group of splits, in order.
  const int per = (nsplit + kCombineGroups - 1) / kCombineGroups;
  const int s0 = warp * per, s1 = min(nsplit, s0 + per);
  float a0 = 0.0f, a1 = 0.0f, l = 0.0f;
#pragma unroll 4
  for (int s = s0; s < s1; s++) {
    const float *ps = pb + s * sstep;
    const float w = expf(__ldcg(ps) - M);
    l = fmaf(__ldcg(ps + 1), w, l);
    a0 = fmaf(__ldcg(ps + 2 + d0 + lane), w, a0);
    if (dims > 32)
      a1 = fmaf(__ldcg(ps + 2 + d0 + 32 + lane), w, a1);
  }
  po[warp][lane] = a0;
  if (dims > 32)
    po[warp][32 + lane] = a1;
  if (lane == 0)
    pl[warp] = l;
  __syncthreads();
  if (tid < dims) {
    float O = po[0][tid], L = pl[0];
    for (int k = 1; k < kCombineGroups; k++) {
      O += po[k][tid];
      L += pl[k];
    }
    const float v = O / L;
    out[r * out_ld + (long long)h * hd + d0 + tid] = v;
    vo[tid] = v;
  }
  if (!oq || dims != gs)
    return;
  __syncthreads();
  if (warp == 0) {
    const float v0 = vo[lane], v1 = dims > 32 ? vo[32 + lane] : 0.0f;
    const int bad = !isfinite(v0) || !isfinite(v1);
    float amax = fmaxf(fabsf(v0), fabsf(v1));
#pragma unroll
    for (int o = 16; o; o >>= 1)
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (__any_sync(0xffffffffu, bad)) {
      if (lane == 0)
        kc_raise(KC_ERR_NONFINITE);
      return;
    }
    const float scl = __fdiv_rn(amax, 127.0f);
    const long long e0 = r * out_ld + (long long)h * hd + d0;
    if (lane == 0)
      os[e0 / gs] = scl;
    oq[e0 + lane] = (int8_t)quantize_value(v0, scl);
    if (dims > 32)
      oq[e0 + 32 + lane] = (int8_t)quantize_value(v1, scl);
  }
}

// Attention for the shapes the split and flash kernels do not take (head_dim not 32, 64 or 128, or more than
// kMaxGqa query heads per KV head), such as the reference's own test fixtures (head_dim 2): one CTA per (query head,
// row) over the row's causal range, the scores in shared memory ([seq] floats). The same softmax as the reference's
// scalar attention: scores q.k / sqrt(head_dim), their maximum, exp(s - max) and its sum, then the weighted values
// divided by the sum; it agrees with the reference within fp32 rounding, as the fast kernels do. Slow by design.
constexpr int kGenericThreads = 256;

__device__ __forceinline__ float block_reduce(float v, float *red, bool is_max) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  __syncthreads();  // red is reused
  if (lane == 0)
    red[warp] = v;
  __syncthreads();
  v = red[0];
  for (int w = 1; w < kGenericThreads / 32; w++)
    v = is_max ? fmaxf(v, red[w]) : v + red[w];
  return v;
}

__global__ void __launch_bounds__(kGenericThreads) attention_generic_kernel(
    float *out, long long out_ld, const float *q, long long q_ld, const float *kc, const float *vc, const int *pos_dev,
    int pos0, int nq, int hd, int seq) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ float sc[];  // [seq]
  __shared__ float red[kGenericThreads / 32];
  const int h = blockIdx.x, r = blockIdx.y, g = h / nq, tid = threadIdx.x;
  const int pos = (pos_dev ? *pos_dev : pos0) + r;
  if (pos < 0 || pos >= seq) {
    if (h == 0 && tid == 0)
      kc_raise(KC_ERR_BAD_ARGS);
    return;
  }
  const int npos = pos + 1;
  const float *qh = q + r * q_ld + (long long)h * hd;
  const float *kh = kc + (long long)g * seq * hd, *vh = vc + (long long)g * seq * hd;
  const float scale = sqrtf((float)hd);
  float mx = -INFINITY;
  for (int t = tid; t < npos; t += kGenericThreads) {
    float s = 0.0f;
    for (int d = 0; d < hd; d++)
      s = fmaf(qh[d], kh[(long long)t * hd + d], s);
    s /= scale;
    sc[t] = s;
    mx = fmaxf(mx, s);
  }
  const float M = block_reduce(mx, red, true);
  float l = 0.0f;
  for (int t = tid; t < npos; t += kGenericThreads) {
    const float e = expf(sc[t] - M);
    sc[t] = e;
    l += e;
  }
  const float L = block_reduce(l, red, false);  // also orders the sc writes above before the reads below
  for (int d = tid; d < hd; d += kGenericThreads) {
    float o = 0.0f;
    for (int t = 0; t < npos; t++)
      o = fmaf(sc[t], vh[(long long)t * hd + d], o);
    out[r * out_ld + (long long)h * hd + d] = o / L;
  }
}

// Shapes the split-K decode and flash prefill kernels take.
bool attention_fast_shape(int n_heads, int n_kv, int hd) {
  return hd % 32 == 0 && hd <= kMaxHd && kAttnThreads % hd == 0 && n_heads / n_kv <= kMaxGqa;
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

int max_splits_for(int seq) { return (seq + kAttnChunk - 1) / kAttnChunk; }

// The generic kernel keeps a row's scores in shared memory: contexts up to 48K positions.
constexpr size_t kGenericMaxSmem = 192 * 1024;

bool attention_shape_ok(const char *name, const AttentionWork *w, int n_heads, int n_kv, int hd, int seq) {
  if (!w || !w->partial)
    return kc_fail("%s: attention work is not initialized", name);
  if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv || hd <= 0 || seq <= 0 ||
      (!attention_fast_shape(n_heads, n_kv, hd) && (size_t)seq * sizeof(float) > kGenericMaxSmem))
    return kc_fail("%s: unsupported heads %d / KV heads %d / head_dim %d / context %d", name, n_heads, n_kv, hd, seq);
  if (n_heads != w->n_heads || hd != w->head_dim || max_splits_for(seq) > w->max_chunks)
    return kc_fail("%s: shape differs from the one the work was initialized for", name);
  return true;
}

// The kernels' dynamic shared-memory limit, raised once per device to what the largest head dimension needs (a limit
// set per call would let a smaller head dimension lower it under a larger one).
bool attention_smem_ready() {
  static bool done[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64)
    return false;
  if (!done[dev]) {
    const int decode = (int)attn_smem_bytes(kMaxHd, kDecodeStages);
    if (cudaFuncSetAttribute(attention_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, decode) ||
        cudaFuncSetAttribute(attention_flash_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)flash_smem_bytes(128)) ||
        cudaFuncSetAttribute(attention_flash_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)flash_smem_bytes(64)) ||
        cudaFuncSetAttribute(attention_flash_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)flash_smem_bytes(32)))
      return false;
    done[dev] = true;
  }
  return true;
}

// One decode row: the split CTAs merge by themselves. Several rows: the row-blocked prefill kernel, then the merge
// kernel, in waves of the work's row capacity. Device positions (graph replay) size the grid for the whole context.
bool attention_rows(const char *name, float *out, long long out_ld, int8_t *oq, float *os, const float *q,
                    long long q_ld, const float *kc, const float *vc, AttentionWork *w, int n_heads, int n_kv, int hd,
                    int seq, const int *pos_dev, int pos0, int rows, int gs) {
  if (!attention_shape_ok(name, w, n_heads, n_kv, hd, seq))
    return false;
  if (oq && (gs <= 0 || (n_heads / n_kv * hd) % gs || out_ld % gs))
    return kc_fail("%s: group size %d does not divide a KV head's outputs", name, gs);
  if (!pos_dev && (pos0 < 0 || pos0 + rows > seq))
    return kc_fail("%s: positions %d..%d outside the context of %d", name, pos0, pos0 + rows - 1, seq);
  if (!attention_smem_ready())
    return kc_fail("%s: cannot reserve %zu bytes of shared memory", name, attn_smem_bytes(hd, kDecodeStages));
  const int max_splits = max_splits_for(seq), nq = n_heads / n_kv;
  if (!attention_fast_shape(n_heads, n_kv, hd)) {
    const size_t smem = (size_t)seq * sizeof(float);
    static bool generic_attr[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !generic_attr[dev]) {
      if (cudaFuncSetAttribute(attention_generic_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kGenericMaxSmem) != cudaSuccess)
        return kc_fail("%s: cannot reserve shared memory for the generic attention", name);
      generic_attr[dev] = true;
    }
    kc_launch_pdl(attention_generic_kernel, dim3(n_heads, rows), kGenericThreads, smem, kc_stream(), out, out_ld, q,
                  q_ld, kc, vc, pos_dev, pos0, nq, hd, seq);
    if (!launched(name))
      return false;
    if (oq) {
      if (kc_launch_quantize_rows(oq, os, out, out_ld, rows, n_heads * hd, gs, kc_stream()) != 0)
        return kc_fail("%s: CUDA launch failed: %s", name, cudaGetErrorString(cudaGetLastError()));
      kc_count_launch();
    }
    return true;
  }
  // Decode CTAs per (KV head, row): one wave of the GPU at two CTAs per SM, never more than the context has chunks.
  int ctas = 2 * kc_device_sms() / n_kv;
  ctas = ctas < 8 ? 8 : ctas;
  // The combine kernel quantizes its block when the block is exactly one quantization group; else a separate pass.
  const int dims = hd < kCombineDims ? hd : kCombineDims;
  const bool fused_q = oq && dims == gs;
  if (rows == 1) {
    // Decode: the split CTAs write one partial per 64-position chunk, the combine kernel merges them.
    const int splits = pos_dev ? max_splits : max_splits_for(pos0 + 1);
    kc_launch_pdl(attention_decode_kernel, dim3(n_kv, ctas < splits ? ctas : splits, 1), kAttnThreads,
                  attn_smem_bytes(hd, kDecodeStages), kc_stream(), q, q_ld, kc, vc, pos_dev, pos0, n_kv, nq, hd, seq,
                  max_splits, w->partial);
    if (!launched(name))
      return false;
    kc_launch_pdl(attention_combine_kernel, dim3(n_heads * (hd / dims), 1), kAttnThreads, 0, kc_stream(), out, out_ld,
                  fused_q ? oq : nullptr, fused_q ? os : nullptr, pos_dev, pos0, n_kv, nq, hd, seq, max_splits,
                  w->partial, gs);
    if (!launched(name))
      return false;
  } else {
    // Prefill: every row of the batch in one flash launch (no partials).
    const dim3 grid(n_kv, (rows + kFlashQ / nq - 1) / (kFlashQ / nq));
    const size_t fsm = flash_smem_bytes(hd);
    if (hd == 128)
      kc_launch_pdl(attention_flash_kernel<128>, grid, kAttnThreads, fsm, kc_stream(), out, out_ld, q, q_ld, kc, vc,
                    pos_dev, pos0, rows, n_kv, nq, seq);
    else if (hd == 64)
      kc_launch_pdl(attention_flash_kernel<64>, grid, kAttnThreads, fsm, kc_stream(), out, out_ld, q, q_ld, kc, vc,
                    pos_dev, pos0, rows, n_kv, nq, seq);
    else
      kc_launch_pdl(attention_flash_kernel<32>, grid, kAttnThreads, fsm, kc_stream(), out, out_ld, q, q_ld, kc, vc,
                    pos_dev, pos0, rows, n_kv, nq, seq);
    if (!launched(name))
      return false;
  }
  if (oq && (rows > 1 || !fused_q)) {
    if (kc_launch_quantize_rows(oq, os, out, out_ld, rows, n_heads * hd, gs, kc_stream()) != 0)
      return kc_fail("%s: CUDA launch failed: %s", name, cudaGetErrorString(cudaGetLastError()));
    kc_count_launch();
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

// ---- attention ----------------------------------------------------------------------------------------------------

// Rows of split-K partials the work holds: the rows asked for, capped by a 512 MiB budget (longer batches run in
// waves), never less than one.
static int attention_work_rows(int n_heads, int head_dim, int seq_len, int rows) {
  const size_t per_row = (size_t)n_heads * max_splits_for(seq_len) * (head_dim + 2) * sizeof(float);
  const size_t fit = ((size_t)512 << 20) / per_row;
  return (int)(fit < 1 ? 1 : fit < (size_t)rows ? fit : (size_t)rows);
}

size_t k_attention_bytes_rows(int n_heads, int n_kv_heads, int head_dim, int seq_len, int rows) {
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || seq_len <= 0 || rows <= 0)
    return 0;
  rows = attention_work_rows(n_heads, head_dim, seq_len, rows);
  const size_t partial = (size_t)rows * n_heads * max_splits_for(seq_len) * (head_dim + 2) * sizeof(float);
  return partial;
}

void k_attention_init_rows(AttentionWork *work, int n_heads, int n_kv_heads, int head_dim, int seq_len, int rows,
                           void *memory) {
  const size_t bytes = k_attention_bytes_rows(n_heads, n_kv_heads, head_dim, seq_len, rows);
  memset(work, 0, sizeof(*work));
  if (!bytes) {
    kc_fail("k_attention_init_rows: invalid shape");
    return;
  }
  rows = attention_work_rows(n_heads, head_dim, seq_len, rows);
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
  work->partial = reinterpret_cast<float *>(base);
  work->max_chunks = max_splits_for(seq_len);
  work->n_heads = n_heads;
  work->head_dim = head_dim;
  work->workers = 1;
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
