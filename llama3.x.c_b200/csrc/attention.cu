// GQA attention over the fp32 head-major K/V cache [kv_head][position][head_dim], in the reference's own arithmetic
// (LucianCrainic/llama3.x.c, src/attention.c), so that it is bitwise the reference's AVX-512 attention:
//  - one row (decode, and a batch of one): the split variant (attention_decode_split, src/attention.c:760-810). The
//    P = position + 1 positions are cut into `chunks` of the team plan (attention_chunks, :516-526), chunk c covering
//    [P c / chunks, P (c + 1) / chunks). Per query head and chunk (attention_chunk_avx512, :40-105): each score is 16
//    lane FMA chains over the head's 16-float vectors, reduced in _mm512_reduce_add_ps's tree, divided by
//    sqrtf(head_dim); the chunk's maximum; exp512 of score - max (the reference's Cephes-style exponential,
//    src/kernels_internal.h:62-76); the exp-sum in 16 lanes (lane l takes positions t0 + 16 i + l) and the same tree;
//    P.V as one FMA chain per output element over the chunk's positions;
//  - a batch of rows: the tiled variant (attention_tiled_avx512 and its driver, :245-334, :1078-1229). Rows form
//    blocks of 16 / (query heads per KV head); a block's chunk length (a multiple of 32) and count come from the plan at
//    its last row. Per query vector and chunk: q scaled once by 1 / sqrtf(head_dim); per 32-position tile the scores as
//    one FMA chain over the head's elements, the tile maximum, and when it exceeds the running one the sum and the
//    accumulator scaled by exp512(old - new); probabilities exp512(score - max); the tile sum as lanes j + 16 + j, then
//    the tree, added to the running sum; P.V as one FMA chain per element over the tile's positions;
//  - both: the chunks merged per head (merge_chunks, :664-682): the maximum over the chunks, then in chunk order
//    sum += w l and o += w acc with w = expf(m - max) (the C library's expf, expf_libc), then o / sum.
// The team plan is the reference's with a team of one (AttentionWork.workers = 1): one chunk per 256 positions, what
// the reference's engine uses whenever its team is no larger than the (local) KV heads.
//
// Kernels: a split CTA per (KV head, chunk) for a row; a tiled CTA per (KV head, group of row blocks) streaming the
// 32-position K/V tiles of the group's causal range (bulk copies, double-buffered) with 64 query vectors on register
// tiles; a merge CTA per (query head, row) that also quantizes the head's outputs for the Wo product. Shapes outside
// the fast kernels (head_dim not 32, 64 or 128, query heads per KV head not dividing 16) run slow one-thread-per-query
// restatements of the same arithmetic.
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>
#include <string.h>

#include "../../include/kernels_cuda.h"
#include "common.cuh"
#include "kernels_cuda_internal.h"

namespace {

constexpr int kTile = 32;        // positions per tile of the batched variant (its TILED_POS)
constexpr int kSplitMax = 256;   // positions of a split chunk at most (attention_chunks' shortest bound)
constexpr int kMaxHd = 256;      // the reference's AVX-512 attention takes head_dim <= 256
constexpr int kMaxNq = 16;       // query heads per KV head (TILED_MAX_Q)
constexpr int kMergeChunks = 16; // chunk partials a merge CTA stages at a time

// ---- the reference's arithmetic, one lane ---------------------------------------------------------------------------

// exp512 (src/kernels_internal.h:62-76) on one lane: the clamp, n = round-to-nearest-even of x * log2(e), the two-step
// reduction by ln 2, the degree-6 Horner polynomial, y * r^2 + (r + 1), then y * 2^n (the result of scalef, one
// rounding: 2^n is exact for n in [-126, 127]; n = 128 goes through y * 2 first, also exact).
__device__ __forceinline__ float exp512_dev(float x) {
  x = fminf(fmaxf(x, -87.33654f), 88.72283f);
  const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(-n, 0.693359375f, x);
  r = __fmaf_rn(-n, -2.12194440e-4f, r);
  float y = 1.9875691500e-4f;
  y = __fmaf_rn(y, r, 1.3981999507e-3f);
  y = __fmaf_rn(y, r, 8.3334519073e-3f);
  y = __fmaf_rn(y, r, 4.1665795894e-2f);
  y = __fmaf_rn(y, r, 1.6666665459e-1f);
  y = __fmaf_rn(y, r, 5.0000001201e-1f);
  y = __fmaf_rn(y, __fmul_rn(r, r), __fadd_rn(r, 1.0f));
  const int ni = (int)n;
  if (ni <= 127)
    return __fmul_rn(y, __int_as_float((ni + 127) << 23));
  return __fmul_rn(__fmul_rn(y, 2.0f), __int_as_float((ni - 1 + 127) << 23));
}


// _mm512_reduce_add_ps over 16 values in registers: halves 8 apart, then 4, then pairs (0, 2) and (1, 3), then the two.
__device__ __forceinline__ float tree16(const float *a) {
  float t8[8], t4[4];
#pragma unroll
  for (int i = 0; i < 8; i++)
    t8[i] = __fadd_rn(a[8 + i], a[i]);
#pragma unroll
  for (int i = 0; i < 4; i++)
    t4[i] = __fadd_rn(t8[4 + i], t8[i]);
  return __fadd_rn(__fadd_rn(t4[0], t4[2]), __fadd_rn(t4[1], t4[3]));
}

// The same tree over a value held by each of 16 consecutive lanes (lane 0 of the 16 gets the result).
__device__ __forceinline__ float tree16_lanes(float v) {
  v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 8, 16));
  v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4, 16));
  v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2, 16));
  return __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1, 16));
}

// attention_chunks (src/attention.c:516-526).
__host__ __device__ inline int plan_chunks(int positions, int n_kv, int limit, int workers) {
  int chunks = (workers + n_kv - 1) / n_kv;
  const int longest = (positions + 31) / 32, shortest = (positions + 255) / 256;
  if (chunks > longest)
    chunks = longest;
  if (chunks < shortest)
    chunks = shortest;
  if (chunks > limit)
    chunks = limit;
  return chunks < 1 ? 1 : chunks;
}

// tiled_plan (src/attention.c:1078-1085): chunk length and count of the block of row `row` (rows counted from the
// batch's first row at pos0, m rows in the batch, `rblock` rows a block).
struct TilePlan {
  int len, chunks;
};
__host__ __device__ inline TilePlan tile_plan(int row, int rblock, int m, int pos0, int n_kv, int limit, int workers) {
  const int block = row / rblock, end = (block + 1) * rblock < m ? (block + 1) * rblock : m;
  const int positions = pos0 + end, wanted = plan_chunks(positions, n_kv, limit, workers);
  TilePlan p;
  p.len = ((positions + wanted - 1) / wanted + kTile - 1) / kTile * kTile;
  p.chunks = (positions + p.len - 1) / p.len;
  return p;
}

__host__ __device__ inline int tile_rblock(int nq) { return 16 / nq < 1 ? 1 : 16 / nq; }

// ---- the partials and their merge ----------------------------------------------------------------------------------
// Partial of (row r of the wave, query head h, chunk c): part[((r * n_heads + h) * cstride + c) * (hd + 2)]:
// the hd accumulator values, then the maximum, then the exp-sum.

// Merges row r's chunks for query head h (blockIdx.x) and writes the head's outputs; with oq, also quantizes them in
// gs-groups (k_quantize's rule) when gs divides head_dim. One thread per output element; every thread walks the
// chunks in order, so all compute the same maximum and sum.
// tiled: the row's plan is its block's (tile_plan), chunks past its visible positions hold nothing and are skipped;
// otherwise (split) the row is the wave's only row and every one of the plan_chunks chunks holds a partial.
__global__ void __launch_bounds__(kMaxHd) merge_kernel(float *out, long long out_ld, int8_t *oq, float *os,
                                                        const float *part, const int *pos_dev, int pos0, int row0,
                                                        int m, int tiled, int n_heads, int n_kv, int hd, int seq,
                                                        int limit, int workers, int cstride, int gs) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[kMaxHd / 32];
  __shared__ float vals[kMaxHd];
  __shared__ float stage[kMergeChunks * (kMaxHd + 2)];
  __shared__ float wts[kMergeChunks];
  const int h = blockIdx.x, rr = blockIdx.y, r = row0 + rr, d = threadIdx.x;
  const int base = pos_dev ? *pos_dev : pos0;
  const int vis = base + r + 1;  // positions the row sees
  if (base < 0 || vis > seq) {
    if (h == 0 && rr == 0 && d == 0)
      kc_raise(KC_ERR_BAD_ARGS);
    return;
  }
  int chunks, live;
  if (tiled) {
    const TilePlan p = tile_plan(r, tile_rblock(n_heads / n_kv), m, base, n_kv, limit, workers);
    chunks = p.chunks;
    live = (vis + p.len - 1) / p.len < chunks ? (vis + p.len - 1) / p.len : chunks;
  } else {
    chunks = plan_chunks(vis, n_kv, limit, workers);
    live = chunks;
  }
  const int slot = hd + 2, nt = blockDim.x;
  const float *pb = part + ((long long)rr * n_heads + h) * cstride * slot;
  // The maximum over the chunks (order-free), every chunk's maximum loaded at once.
  float mx = -FLT_MAX;
  for (int c = d; c < live; c += nt)
    mx = fmaxf(mx, __ldcg(pb + (long long)c * slot + hd));
#pragma unroll
  for (int off = 16; off; off >>= 1)
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((d & 31) == 0)
    red[d >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < nt / 32; w++)
    mx = fmaxf(mx, red[w]);
  // Then the chunks in order, kMergeChunks at a time staged in shared memory by one round of parallel loads; each
  // chunk's weight is taken once, and every thread adds the sums in chunk order.
  float sum = 0.0f, o = 0.0f;
  for (int c0 = 0; c0 < live; c0 += kMergeChunks) {
    const int nc = min(kMergeChunks, live - c0);
    __syncthreads();  // the previous block's reads are done (and red's, above)
    for (int i = d; i < nc * slot; i += nt)
      stage[i] = __ldcg(pb + (long long)c0 * slot + i);
    __syncthreads();
    if (d < nc)
      wts[d] = expf_libc(__fsub_rn(stage[d * slot + hd], mx));
    __syncthreads();
    for (int c = 0; c < nc; c++) {
      const float w = wts[c];
      sum = __fadd_rn(sum, __fmul_rn(w, stage[c * slot + hd + 1]));
      if (d < hd)
        o = __fadd_rn(o, __fmul_rn(w, stage[c * slot + d]));
    }
  }
  (void)chunks;
  const float v = __fdiv_rn(o, sum);
  float *dst = out + (long long)r * out_ld + (long long)h * hd;
  if (d < hd)
    dst[d] = v;
  if (!oq || gs <= 0 || hd % gs)
    return;
  // Quantize the head's outputs group by group: the group maximum of |v| (order-free), scale = max / 127.
  const int warp = d >> 5, lane = d & 31;
  vals[d] = v;
  const int bad = d < hd && !isfinite(v);
  float a = d < hd ? fabsf(v) : 0.0f;
  if (__syncthreads_or(bad)) {
    if (d == 0)
      kc_raise(KC_ERR_NONFINITE);
    return;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1)
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
  if (lane == 0)
    red[warp] = a;
  __syncthreads();
  if (d < hd) {
    const int g0 = (d / gs) * gs, w0 = g0 >> 5, w1 = (g0 + gs - 1) >> 5;
    float gmax = 0.0f;
    if (gs >= 32) {
      for (int w = w0; w <= w1; w++)
        gmax = fmaxf(gmax, red[w]);
    } else {
      for (int i = g0; i < g0 + gs; i++)
        gmax = fmaxf(gmax, fabsf(vals[i]));
    }
    const float scl = __fdiv_rn(gmax, 127.0f);
    const long long e = (long long)r * out_ld + (long long)h * hd + d;
    oq[e] = (int8_t)quantize_value(v, scl);
    if (d == g0)
      os[e / gs] = scl;
  }
}

// merge_chunks for one (row, query head) by one warp: lane c takes chunk c's maximum, weight and weighted sum (the sum
// then runs over the chunks in order through shuffles), and each lane adds up hd / 32 elements over the chunks in
// order, eight chunks' values in flight at a time. pb: the head's chunk partials (slot hd + 2 floats apart), `live`
// of them; dst: its hd outputs; with oq, the outputs are also quantized in gs-groups (group maxima by shuffles over
// the gs / (hd / 32) lanes that hold a group; merge_warp_quantizes) into oq[e0 ..] and os[e0 / gs ..], e0 being the
// outputs' element index. Returns false (the error raised) when an output is not finite, before quantizing.
template <int HD>
__device__ bool merge_head_warp(const float *pb, int live, float *dst, int8_t *oq, float *os, long long e0, int gs) {
  constexpr int DL = HD / 32, slot = HD + 2;
  const int lane = threadIdx.x & 31;
  // One round of loads covers the common case: lane c's chunk maximum and sum (chunks < 32) and the first eight
  // chunks' elements, all in flight together; only the maxima of chunks 32.. and the elements of chunks 8.. follow.
  float m0 = -FLT_MAX, l0 = 0.0f, a[8][DL];
  if (lane < live) {
    m0 = __ldcg(pb + (long long)lane * slot + HD);
    l0 = __ldcg(pb + (long long)lane * slot + HD + 1);
  }
#pragma unroll
  for (int u = 0; u < 8; u++)
#pragma unroll
    for (int e = 0; e < DL; e++)
      a[u][e] = u < live ? __ldcg(pb + (long long)u * slot + DL * lane + e) : 0.0f;
  float mx = fmaxf(-FLT_MAX, m0);
  for (int c = lane + 32; c < live; c += 32)
    mx = fmaxf(mx, __ldcg(pb + (long long)c * slot + HD));
#pragma unroll
  for (int off = 16; off; off >>= 1)
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  float sum = 0.0f, o[DL];
#pragma unroll
  for (int e = 0; e < DL; e++)
    o[e] = 0.0f;
  for (int c0 = 0; c0 < live; c0 += 32) {
    float w = 0.0f, wl = 0.0f;
    if (c0 + lane < live) {
      const float *pc = pb + (long long)(c0 + lane) * slot;
      const float mc = c0 == 0 ? m0 : __ldcg(pc + HD), lc = c0 == 0 ? l0 : __ldcg(pc + HD + 1);
      w = expf_libc(__fsub_rn(mc, mx));
      wl = __fmul_rn(w, lc);
    }
    const int nb = min(32, live - c0);
    for (int i = 0; i < nb; i += 8) {
      if (c0 > 0 || i > 0) {
#pragma unroll
        for (int u = 0; u < 8; u++)
#pragma unroll
          for (int e = 0; e < DL; e++)
            a[u][e] = i + u < nb ? __ldcg(pb + (long long)(c0 + i + u) * slot + DL * lane + e) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const float wc = __shfl_sync(0xffffffffu, w, (i + u) & 31), wlc = __shfl_sync(0xffffffffu, wl, (i + u) & 31);
        if (i + u < nb) {
          sum = __fadd_rn(sum, wlc);
#pragma unroll
          for (int e = 0; e < DL; e++)
            o[e] = __fadd_rn(o[e], __fmul_rn(wc, a[u][e]));
        }
      }
    }
  }
  float v[DL];
  bool bad = false;
#pragma unroll
  for (int e = 0; e < DL; e++) {
    v[e] = __fdiv_rn(o[e], sum);
    dst[DL * lane + e] = v[e];
    bad |= !isfinite(v[e]);
  }
  if (!oq)
    return true;
  if (__any_sync(0xffffffffu, bad)) {
    if (lane == 0)
      kc_raise(KC_ERR_NONFINITE);
    return false;
  }
  // Group maximum of |v| over the gs / DL lanes that hold the group (order-free), scale = max / 127.
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < DL; e++)
    amax = fmaxf(amax, fabsf(v[e]));
  for (int off = gs / DL / 2; off; off >>= 1)
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float scl = __fdiv_rn(amax, 127.0f);
  const long long el = e0 + DL * lane;
#pragma unroll
  for (int e = 0; e < DL; e++)
    oq[el + e] = (int8_t)quantize_value(v[e], scl);
  if ((DL * lane) % gs == 0)
    os[el / gs] = scl;
  return true;
}

// The merge of a batch of rows on the fast shapes, a warp per (row, query head) (merge_head_warp), so no CTA-wide
// step remains. Quantizes only when merge_warp_quantizes(hd, gs).
template <int HD>
__global__ void __launch_bounds__(256) merge_warp_kernel(float *out, long long out_ld, int8_t *oq, float *os,
                                                         const float *part, const int *pos_dev, int pos0, int row0,
                                                         int m, int wave, int n_heads, int n_kv, int seq, int limit,
                                                         int workers, int cstride, int gs) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, pair = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (pair >= wave * n_heads)
    return;
  const int rr = pair / n_heads, h = pair - rr * n_heads, r = row0 + rr;
  const int base = pos_dev ? *pos_dev : pos0;
  const int vis = base + r + 1;  // positions the row sees
  if (base < 0 || vis > seq) {
    if (pair == 0 && lane == 0)
      kc_raise(KC_ERR_BAD_ARGS);
    return;
  }
  const TilePlan p = tile_plan(r, tile_rblock(n_heads / n_kv), m, base, n_kv, limit, workers);
  const int live = min((vis + p.len - 1) / p.len, p.chunks);  // chunks past the visible positions hold nothing
  const long long e0 = (long long)r * out_ld + (long long)h * HD;
  merge_head_warp<HD>(part + ((long long)rr * n_heads + h) * cstride * (HD + 2), live, out + e0, oq, os, e0, gs);
}

// ---- slow restatements for the shapes the fast kernels do not take --------------------------------------------------

// One thread per (query head, chunk) of one row: attention_chunk_avx512 (src/attention.c:40-105) for head_dim <= 256.
__global__ void split_generic_kernel(const float *q, const float *kc, const float *vc, const int *pos_dev, int pos0,
                                     int n_heads, int n_kv, int hd, int seq, int limit, int workers, int cstride,
                                     float *part) {
  pdl_wait();
  pdl_launch_dependents();
  const int h = blockIdx.x, c = threadIdx.x;
  const int P = (pos_dev ? *pos_dev : pos0) + 1;
  if (P < 1 || P > seq)
    return;  // the merge kernel reports it
  const int chunks = plan_chunks(P, n_kv, limit, workers);
  if (c >= chunks)
    return;
  const int t0 = (int)((long long)P * c / chunks), t1 = (int)((long long)P * (c + 1) / chunks);
  const int g = h / (n_heads / n_kv), vectors = (hd + 15) / 16;
  const float *qh = q + (long long)h * hd, *K = kc + (long long)g * seq * hd, *V = vc + (long long)g * seq * hd;
  float *o = part + ((long long)h * cstride + c) * (hd + 2);
  const float divisor = __fsqrt_rn((float)hd);
  // Pass 1: the maximum score. Pass 2: exp-sum lanes. Pass 3: P.V per element (scores recomputed each pass).
  auto score = [&](int t) {
    float lanes[16];
    for (int l = 0; l < 16; l++)
      lanes[l] = 0.0f;
    for (int v = 0; v < vectors; v++)
      for (int l = 0; l < 16 && 16 * v + l < hd; l++)
        lanes[l] = __fmaf_rn(qh[16 * v + l], K[(long long)t * hd + 16 * v + l], lanes[l]);
    return __fdiv_rn(tree16(lanes), divisor);
  };
  float mx = -FLT_MAX;
  for (int t = t0; t < t1; t++)
    mx = fmaxf(mx, score(t));
  float vsum[16];
  for (int l = 0; l < 16; l++)
    vsum[l] = 0.0f;
  for (int t = t0; t < t1; t++)
    vsum[(t - t0) & 15] = __fadd_rn(vsum[(t - t0) & 15], exp512_dev(__fsub_rn(score(t), mx)));
  for (int d = 0; d < hd; d++)
    o[d] = 0.0f;
  for (int t = t0; t < t1; t++) {
    const float e = exp512_dev(__fsub_rn(score(t), mx));
    for (int d = 0; d < hd; d++)
      o[d] = __fmaf_rn(e, V[(long long)t * hd + d], o[d]);
  }
  o[hd] = mx;
  o[hd + 1] = tree16(vsum);
}

// One thread per (query head, row, chunk) of a batch: attention_tiled_avx512 (src/attention.c:245-334) for one query
// vector, head_dim <= 256. The accumulator lives in the partial itself.
__global__ void tiled_generic_kernel(const float *q, long long q_ld, const float *kc, const float *vc, int pos0,
                                     int row0, int rows, int m, int n_heads, int n_kv, int hd, int seq, int limit,
                                     int workers, int cstride, float *part) {
  pdl_wait();
  pdl_launch_dependents();
  const int h = blockIdx.x, rr = blockIdx.y, c = threadIdx.x, r = row0 + rr;
  if (rr >= rows)
    return;
  const int nq = n_heads / n_kv, g = h / nq, vis = pos0 + r + 1;
  const TilePlan p = tile_plan(r, tile_rblock(nq), m, pos0, n_kv, limit, workers);
  const int t0 = c * p.len, t1 = min((c + 1) * p.len, vis);
  if (c >= p.chunks || t1 <= t0)
    return;  // nothing visible: the merge skips the chunk
  const float *qh = q + (long long)r * q_ld + (long long)h * hd, *K = kc + (long long)g * seq * hd,
              *V = vc + (long long)g * seq * hd;
  float *o = part + (((long long)rr * n_heads + h) * cstride + c) * (hd + 2);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  float m_run = -FLT_MAX, l = 0.0f;
  for (int d = 0; d < hd; d++)
    o[d] = 0.0f;
  for (int t = t0; t < t1; t += kTile) {
    const int n = min(kTile, t1 - t);
    float s[kTile], e[kTile];
    for (int j = 0; j < n; j++) {
      float a = 0.0f;
      for (int d = 0; d < hd; d++)
        a = __fmaf_rn(__fmul_rn(qh[d], scale), K[(long long)(t + j) * hd + d], a);
      s[j] = a;
    }
    float tmax = -FLT_MAX;
    for (int j = 0; j < n; j++)
      tmax = fmaxf(tmax, s[j]);
    if (tmax > m_run) {
      const float alpha = exp512_dev(__fsub_rn(m_run, tmax));
      l = __fmul_rn(l, alpha);
      for (int d = 0; d < hd; d++)
        o[d] = __fmul_rn(o[d], alpha);
      m_run = tmax;
    }
    for (int j = 0; j < kTile; j++)
      e[j] = j < n ? exp512_dev(__fsub_rn(s[j], m_run)) : 0.0f;
    float lanes[16];
    for (int j = 0; j < 16; j++)
      lanes[j] = __fadd_rn(e[j], e[16 + j]);
    l = __fadd_rn(l, tree16(lanes));
    for (int j = 0; j < n; j++)
      for (int d = 0; d < hd; d++)
        o[d] = __fmaf_rn(e[j], V[(long long)(t + j) * hd + d], o[d]);
  }
  o[hd] = m_run;
  o[hd + 1] = l;
}

// ---- the split variant for one row (decode) -----------------------------------------------------------------------
// A cluster of kSplitCtas CTAs per (KV head g, chunk c) of the row at position pos: CTA k of the cluster loads K rows
// [k n / 4, (k + 1) n / 4) of the chunk's n <= 256 positions (one bulk copy) and V[chunk rows][its quarter of the
// head's elements] (cp.async), computes the scores of its K rows for the group's nq heads and stores each into the
// score buffer of every CTA of the cluster through distributed shared memory, so that after one cluster barrier each
// CTA holds all of the chunk's scores. Each CTA then takes the maximum, exp512 and the 16-lane exp-sum per head
// (the same in every CTA) and runs the P.V chains of its quarter of the head's elements. So each K and V element is
// read once. A cluster walks chunks y, y + gridDim.y, ... (about one wave of clusters). With `tickets`, the CTA that
// finishes a KV head's last chunk also merges the group's partials (the arithmetic of merge_kernel) and writes its
// outputs, so no second launch waits on the partials.
// With `early` (the position read from device memory), the K and V rows below the newest position are requested
// before the wait on the preceding kernel: the caller guarantees that the launch before this one writes neither the
// position word nor any cache row below it (a decode step's K/V store writes only the newest row), so those copies
// overlap the preceding kernel's tail. The newest row, Q and everything else is read after the wait.
constexpr int kSplitCtas = 4;
constexpr int kSplitThreads = 256;
constexpr int kSplitTickets = 256;  // KV heads the fused merge serves (a ticket word each, past the partials)
constexpr int kSplitRows = kSplitMax / kSplitCtas;  // K rows of a CTA at most

// Floats before the mbarrier: K quarter [kSplitRows][hd], V quarter [kSplitMax][hd / 4], Q [nq][hd], the chunk's
// scores (then probabilities) [nq][kSplitMax], which every CTA of the cluster writes its rows into, the per-head
// maximum and exp-sum.
__host__ __device__ constexpr size_t split_smem_floats(int hd, int nq) {
  return (size_t)kSplitRows * hd + (size_t)kSplitMax * (hd / kSplitCtas) + (size_t)nq * hd + (size_t)nq * kSplitMax +
         2 * kMaxNq;
}
__host__ __device__ constexpr size_t split_smem_bytes(int hd, int nq) {
  return split_smem_floats(hd, nq) * sizeof(float) + sizeof(uint64_t);
}

__device__ __forceinline__ void st_cluster_u32(unsigned *local, unsigned rank, unsigned v) {
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(remote), "r"(v) : "memory");
}

__device__ __forceinline__ void st_cluster_f32(float *local, unsigned rank, float v) {
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}


__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// One butterfly step of the 16-lane tree over W positions at once: the lane keeps the half of its positions whose
// bit `off` matches its own and adds its partner's copy of them (a + b is b + a, so both lanes of a pair agree with
// the tree's operand order).
template <int W>
__device__ __forceinline__ void tree_step(const float *in, float *outv, int L, int off) {
  const bool hi = L & off;
#pragma unroll
  for (int i = 0; i < W / 2; i++) {
    const float send = hi ? in[i] : in[W / 2 + i], keep = hi ? in[W / 2 + i] : in[i];
    outv[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, off));
  }
}

// Group g's merge by the CTA that finished its last chunk: merge_kernel's arithmetic (the maximum over the chunks, then
// in chunk order sum += w l and o += w acc with w = expf(m_c - max), then o / sum, then the optional quantization),
// a warp per query head of the group (merge_head_warp).
template <int HD>
__device__ void merge_group(const float *part, int g, int nq, int chunks, int cstride, float *out, int8_t *oq,
                            float *os, int gs) {
  for (int hh = threadIdx.x >> 5; hh < nq; hh += kSplitThreads / 32) {
    const long long e0 = (long long)(g * nq + hh) * HD;
    merge_head_warp<HD>(part + (long long)(g * nq + hh) * cstride * (HD + 2), chunks, out + e0, oq, os, e0, gs);
  }
}

// The decode step's RoPE and K/V store folded into the split kernel (k_rope_attention_q8_step): q, k, v are the QKV
// product of the newest position, unrotated; the kernel rotates q and k with the table row of that position as
// rope_store_kernel does, uses the newest row from registers instead of the cache, and writes it into the caches
// (kc, vc) for the positions after it. table == nullptr: off (q is then the rotated queries, the caches complete).
struct RopeStep {
  const float *k, *v, *table;
  float *kc, *vc;
};

// K rows [r0, r1) of the chunk starting at position t0 into this CTA's K quarter (its first row k0), one bulk copy.
template <int HD>
__device__ __forceinline__ void split_copy_k(float *Kq, const float *Kh, uint64_t *bar, int t0, int k0, int r0,
                                             int r1) {
  if (threadIdx.x == 0 && r1 > r0)
    bulk_g2s(Kq + (long long)(r0 - k0) * HD, Kh + (long long)(t0 + r0) * HD, (unsigned)(r1 - r0) * HD * 4, bar);
}

// V rows [r0, r1) of the chunk, the columns of CTA k's quarter, as 16-byte cp.async pieces.
template <int HD>
__device__ __forceinline__ void split_copy_v(float *Vq, const float *Vh, int t0, int k, int r0, int r1) {
  constexpr int QD = HD / kSplitCtas, PR = QD / 4;
  for (int i = threadIdx.x; i < (r1 - r0) * PR; i += kSplitThreads) {
    const int t = r0 + i / PR, p4 = i % PR;
    cp_async16(Vq + t * QD + 4 * p4, Vh + (long long)(t0 + t) * HD + k * QD + 4 * p4);
  }
}

template <int HD>
__global__ void __launch_bounds__(kSplitThreads, 3) split_kernel(const float *q, const float *kc, const float *vc,
                                                              const int *pos_dev, int pos0, int n_kv, int nq, int seq,
                                                              int limit, int workers, int cstride, float *part,
                                                              unsigned *tickets, float *out, int8_t *oq, float *os,
                                                              int gs, int early, const RopeStep rope) {
  constexpr int QD = HD / kSplitCtas;  // elements of the head this CTA's P.V covers
  extern __shared__ __align__(16) float sm[];
  float *Kq = sm, *Vq = Kq + kSplitRows * HD, *Q = Vq + kSplitMax * QD, *S = Q + nq * HD;
  float *hmax = S + nq * kSplitMax, *hsum = hmax + kMaxNq;
  uint64_t *bar = reinterpret_cast<uint64_t *>(sm + split_smem_floats(HD, nq));
  __shared__ unsigned fails[kSplitCtas];
  __shared__ int last;
  static_assert(kSplitCtas == 4, "the failure vote reads four slots");
  const int g = blockIdx.x, k = blockIdx.z, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  bool waited = !early;
  if (waited) {
    pdl_wait();
    pdl_launch_dependents();
  }
  const int P = (pos_dev ? *pos_dev : pos0) + 1;
  if (P < 1 || P > seq) {  // every CTA of the cluster leaves here together
    if (tickets && g == 0 && blockIdx.y == 0 && k == 0 && tid == 0)
      kc_raise(KC_ERR_BAD_ARGS);  // (without tickets the merge kernel reports it)
    return;
  }
  const int chunks = plan_chunks(P, n_kv, limit, workers);
  if ((int)blockIdx.y >= chunks)
    return;  // likewise together
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int newest = P - 1;  // the only cache row the preceding launch may write (early mode)
  const float *Kh = kc + (long long)g * seq * HD, *Vh = vc + (long long)g * seq * HD;
  // The cluster walks chunks blockIdx.y, blockIdx.y + gridDim.y, ...; every CTA of it takes the same steps.
  unsigned phase = 0;
  for (int c = blockIdx.y; c < chunks; c += gridDim.y) {
    const int t0 = (int)((long long)P * c / chunks), n = (int)((long long)P * (c + 1) / chunks) - t0;  // <= 256
    const int k0 = n * k / kSplitCtas, kn = n * (k + 1) / kSplitCtas - k0;  // this CTA's K rows
    // Rows [t0 + r0, t0 + r1) of K (this CTA's) and V (the whole chunk, this CTA's columns); before the wait only
    // those below the newest row. With the RoPE step the newest row comes from the QKV product instead (new_k: it
    // is one of this CTA's K rows), and Q is rotated here rather than copied.
    const bool rope_on = rope.table != nullptr, has_new = rope_on && newest - t0 < n;
    const bool new_k = has_new && newest - t0 >= k0 && newest - t0 < k0 + kn;
    if (tid == 0)
      mbar_arrive_expect_tx(bar, (unsigned)(kn - (new_k ? 1 : 0) + (rope_on ? 0 : nq)) * HD * sizeof(float));
    const int below_new = min(n, max(0, newest - t0));
    const int split_at = rope_on || !waited ? below_new : n;  // chunk rows to copy now (the RoPE step: ever)
    split_copy_k<HD>(Kq, Kh, bar, t0, k0, k0, min(k0 + kn, max(k0, split_at)));
    split_copy_v<HD>(Vq, Vh, t0, k, 0, split_at);
    if (!waited) {
      pdl_wait();
      pdl_launch_dependents();
      waited = true;
      if (!rope_on) {
        split_copy_k<HD>(Kq, Kh, bar, t0, k0, max(k0, split_at), k0 + kn);
        split_copy_v<HD>(Vq, Vh, t0, k, split_at, n);
      }
    }
    if (!rope_on) {
      if (tid == 0)  // the group's queries (written by the previous kernel: after the wait)
        bulk_g2s(Q, q + (long long)g * nq * HD, (unsigned)nq * HD * sizeof(float), bar);
    } else {
      // rope_store_kernel's rotation of the pairs (j, j + 1) with the newest position's table row.
      const float *tr = rope.table + (long long)newest * 2 * HD;
      for (int i = tid; i < nq * HD / 2; i += kSplitThreads) {
        const int h = i / (HD / 2), j = 2 * (i - h * (HD / 2));
        const float *src = q + (long long)(g * nq + h) * HD + j;
        const float cs = tr[j], sn = tr[HD + j + 1], a0 = src[0], b0 = src[1];
        Q[h * HD + j] = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(b0, sn));
        Q[h * HD + j + 1] = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(b0, cs));
      }
      if (has_new) {
        const float *kr = rope.k + (long long)g * HD, *vr = rope.v + (long long)g * HD;
        float *kcw = rope.kc + ((long long)g * seq + newest) * HD, *vcw = rope.vc + ((long long)g * seq + newest) * HD;
        for (int i = tid; i < HD / 2; i += kSplitThreads) {
          const int j = 2 * i;
          const float cs = tr[j], sn = tr[HD + j + 1], a0 = kr[j], b0 = kr[j + 1];
          const float o0 = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(b0, sn));
          const float o1 = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(b0, cs));
          if (new_k)
            Kq[(newest - t0 - k0) * HD + j] = o0, Kq[(newest - t0 - k0) * HD + j + 1] = o1;
          if (k == 0)  // the cache row, for the positions after this one
            kcw[j] = o0, kcw[j + 1] = o1;
        }
        for (int i = tid; i < QD; i += kSplitThreads)
          Vq[(newest - t0) * QD + i] = vr[k * QD + i];
        if (k == 0)
          for (int i = tid; i < HD; i += kSplitThreads)
            vcw[i] = vr[i];
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    const bool ok = __syncthreads_and(mbar_wait_bounded(bar, phase));
    phase ^= 1u;
    if (ok) {
      // Scores: a warp per (16 positions, 2 heads), a half-warp per head, lane L the reference's lane L (its FMA
      // chain over elements 16 v + L); the 16-lane tree of all 16 positions runs as one butterfly, after which lane
      // L holds position L's score.
      const int hw = lane >> 4, L = lane & 15, groups = (kn + 15) >> 4, pairs = (nq + 1) >> 1;
      const float divisor = __fsqrt_rn((float)HD);
      for (int task = warp; task < groups * pairs; task += kSplitThreads / 32) {
        const int grp = task % groups, h = (task / groups) * 2 + hw, hc = h < nq ? h : nq - 1;
        float qv[HD / 16];
#pragma unroll
        for (int v = 0; v < HD / 16; v++)
          qv[v] = Q[hc * HD + 16 * v + L];
        int row[16];
#pragma unroll
        for (int j = 0; j < 16; j++)
          row[j] = (grp * 16 + j < kn ? grp * 16 + j : kn - 1) * HD + L;
        float a16[16];
#pragma unroll
        for (int j = 0; j < 16; j++)
          a16[j] = 0.0f;
#pragma unroll
        for (int v = 0; v < HD / 16; v++)
#pragma unroll
          for (int j = 0; j < 16; j++)
            a16[j] = __fmaf_rn(qv[v], Kq[row[j] + 16 * v], a16[j]);
        float t8[8], t4[4], t2[2], t1[1];
        tree_step<16>(a16, t8, L, 8);
        tree_step<8>(t8, t4, L, 4);
        tree_step<4>(t4, t2, L, 2);
        tree_step<2>(t2, t1, L, 1);
        const int t = grp * 16 + L;
        if (h < nq && t < kn) {
          // Position k0 + t of the chunk: into the scores of every CTA of the cluster (its own included), so the
          // barrier below leaves each with all of the chunk's scores and nothing has to be fetched afterwards.
          const float sc = __fdiv_rn(t1[0], divisor);
#pragma unroll
          for (int r = 0; r < kSplitCtas; r++)
            st_cluster_f32(S + h * kSplitMax + k0 + t, (unsigned)r, sc);
        }
      }
    } else if (tid == 0) {
      mbar_wait_bounded(bar, phase ^ 1u);  // let the copy in flight land (bounded) before leaving
    }
    // Each CTA's verdict (uniform within it) into slot k of every CTA, so that all of them see one failure.
    if (tid < kSplitCtas)
      st_cluster_u32(fails + k, (unsigned)tid, ok ? 0u : 1u);
    cluster_sync_all();  // every CTA of the cluster arrives, whatever happened above
    if (fails[0] | fails[1] | fails[2] | fails[3]) {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
      cluster_sync_all();  // no CTA leaves while another may still read its scores
      break;             // the whole cluster stops in the same iteration (the error is raised)
    }
    // Per head (a warp each): the maximum, exp512, the exp-sum in 16 lanes (lane l adds positions l, l + 16, l + 32,
    // ... in order: l + 32 i is its own value i, l + 16 + 32 i lane l + 16's) then the tree.
    for (int h = warp; h < nq; h += kSplitThreads / 32) {
      float *sh = S + h * kSplitMax;
      float sv[kSplitMax / 32];
      float mx = -FLT_MAX;
#pragma unroll
      for (int i = 0; i < kSplitMax / 32; i++) {
        const int t = lane + 32 * i;
        sv[i] = t < n ? sh[t] : -FLT_MAX;
        mx = fmaxf(mx, sv[i]);
      }
#pragma unroll
      for (int off = 16; off; off >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      float vs = 0.0f;
#pragma unroll
      for (int i = 0; i < kSplitMax / 32; i++) {
        const int t = lane + 32 * i;
        const float e = t < n ? exp512_dev(__fsub_rn(sv[i], mx)) : 0.0f;
        if (t < n)
          sh[t] = e;
        const float hi = __shfl_down_sync(0xffffffffu, e, 16);
        if (t < n)
          vs = __fadd_rn(vs, e);
        if (t + 16 < n)
          vs = __fadd_rn(vs, hi);
      }
      vs = tree16_lanes(vs);
      if (lane == 0)
        hmax[h] = mx, hsum[h] = vs;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // P.V: a chain per (head, element of this CTA's quarter) over the chunk's positions in order; the next eight
    // positions' operands are loaded while the current eight are added.
    for (int i = tid; i < nq * QD; i += kSplitThreads) {
      const int h = i / QD, d = i - h * QD;
      const float *e = S + h * kSplitMax, *vd = Vq + d;
      float acc = 0.0f;
      float ea[8], va[8];
#pragma unroll
      for (int u = 0; u < 8; u++)
        ea[u] = e[u], va[u] = vd[u * QD];
      int t = 0;
      for (; t + 8 <= n; t += 8) {
        float eb[8], vb[8];
#pragma unroll
        for (int u = 0; u < 8; u++)
          eb[u] = e[t + 8 + u], vb[u] = vd[(t + 8 + u) * QD];  // (reads past n stay inside shared memory)
#pragma unroll
        for (int u = 0; u < 8; u++)
          acc = __fmaf_rn(ea[u], va[u], acc);
#pragma unroll
        for (int u = 0; u < 8; u++)
          ea[u] = eb[u], va[u] = vb[u];
      }
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (t + u < n)
          acc = __fmaf_rn(ea[u], va[u], acc);
      part[((long long)(g * nq + h) * cstride + c) * (HD + 2) + k * QD + d] = acc;
    }
    if (k == 0 && tid < nq) {
      float *o = part + ((long long)(g * nq + tid) * cstride + c) * (HD + 2);
      o[HD] = hmax[tid];
      o[HD + 1] = hsum[tid];
    }
    // The scores, K and V buffers are refilled by the cluster's next chunk, whose scores the other CTAs write into
    // this CTA's buffer: every CTA is done with them first. After the cluster's last chunk no CTA touches another's
    // shared memory any more (the scores were exchanged before the barrier above), so none waits.
    if (c + (int)gridDim.y < chunks)
      cluster_sync_all();
  }
  if (!tickets)
    return;
  // Every CTA that took chunks counts them (after a failure too, so the count stays whole); the one that completes
  // the KV head's 4 x chunks merges it and resets the ticket for the next call.
  const unsigned mine = (unsigned)((chunks - 1 - (int)blockIdx.y) / (int)gridDim.y + 1);
  __syncthreads();
  if (tid == 0) {
    // One acquire-release add: it publishes this CTA's partials (written before the barrier above) and, for the CTA
    // that completes the count, makes every other CTA's partials visible to the merge after the barrier below. The
    // reset is read by the next call, a later kernel.
    unsigned before;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(before) : "l"(tickets + g), "r"(mine) : "memory");
    last = before + mine == (unsigned)(kSplitCtas * chunks);
    if (last)
      tickets[g] = 0u;
  }
  __syncthreads();
  if (last)
    merge_group<HD>(part, g, nq, chunks, cstride, out, oq, os, gs);
}

// ---- the tiled variant for a batch of rows (prefill) ---------------------------------------------------------------
// CTA (KV head g, group of R rows = whole blocks): its query vectors v = (row - first row) * nq + head, at most 128,
// over the 32-position K/V tiles of the group's causal range (bulk copies, two buffers, the next tile's copy in
// flight; K rows padded in shared memory so that rows read together sit in different banks). Warp w owns query
// vectors 16 w .. 16 w + 15 from the scores to the P.V product, so within a tile its warps never wait for one another
// (8 warps, two per SM sub-partition: with 16 queries a warp, 4 x 4 scores a lane take 8 operand reads per 64 FMAs
// where 2 x 4 took 6 per 32, and P.V's probabilities are warp-wide broadcasts):
//  - scores: lane (lv, lp) = (lane / 8, lane % 8) takes queries 16 w + lv + 4 i (i < 4) and positions lp + 8 j
//    (j < 4), each score one FMA chain over the head's elements in order, operands read four elements at a time;
//  - the online softmax of the tile for each query, among the 8 lanes that share it: the tile maximum, the rescale of
//    the running sum, exp512, and the tile sum in the reference's order (positions p and 16 + p are the same lane's
//    j and j + 2, then the 16-lane tree by shuffles across the 8 lanes); every lane keeps the queries' running
//    maximum, sum and chunk;
//  - P.V: every lane takes the warp's 16 queries x hd / 32 elements, one FMA chain per (query, element) over the
//    tile's positions in order; the probabilities are read as warp-wide broadcasts.
// A query whose chunk (its block's plan) changes at a tile writes the finished chunk's partial first and starts again
// from zero. The partials are merged by merge_kernel.
constexpr int kTQ = 128;            // query vectors of a batched CTA
constexpr int kQW = 16;             // query vectors of a warp
constexpr int kQL = kQW / 4;        // query vectors of a lane in the score role
constexpr int kTWarps = kTQ / kQW;  // 8 warps
constexpr int kPStride = kTQ + 4;   // probabilities [tile position][query vector], padded

__host__ __device__ constexpr int tiled_kstride(int hd) { return hd + 4; }  // padded K and Q rows
__host__ __device__ constexpr size_t tiled_smem_bytes(int hd) {
  return ((size_t)kTQ * tiled_kstride(hd) + 2 * (size_t)kTile * tiled_kstride(hd) + 2 * (size_t)kTile * hd +
          (size_t)kTile * kPStride + 2 * kTQ) * sizeof(float) + 2 * sizeof(uint64_t);
}

template <int HD>
__global__ void __launch_bounds__(kTWarps * 32, 1) tiled_kernel(const float *q, long long q_ld, const float *kc,
                                                             const float *vc, const int *pos_dev, int pos0, int row0,
                                                             int rows, int m, int R, int n_kv, int nq, int seq,
                                                             int limit, int workers, int cstride, float *part) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int KS = tiled_kstride(HD), DL = HD / 32;  // padded row; P.V elements of a lane
  extern __shared__ __align__(16) float sm[];
  float *qs = sm, *Kb = qs + kTQ * KS, *Vb = Kb + 2 * kTile * KS, *P = Vb + 2 * kTile * HD, *al = P + kTile * kPStride;
  int *fl = reinterpret_cast<int *>(al + kTQ);
  uint64_t *bar = reinterpret_cast<uint64_t *>(fl + kTQ);
  const int g = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int base = pos_dev ? *pos_dev : pos0;
  // Row groups in reverse order: the longest causal ranges start first.
  const int rl0 = (gridDim.y - 1 - blockIdx.y) * R, nr = min(R, rows - rl0);  // rows of this CTA, from wave row rl0
  if (nr <= 0 || base < 0 || base + row0 + rl0 + nr > seq)
    return;  // the merge kernel reports bad positions
  const int qv = nr * nq, rblock = tile_rblock(nq), n_heads = n_kv * nq;
  const int vis_max = base + row0 + rl0 + nr, ntiles = (vis_max + kTile - 1) / kTile;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  // Queries, scaled: qs[v][d].
  for (int i = tid; i < kTQ * HD; i += kTWarps * 32) {
    const int v = i / HD, d = i - v * HD;
    float x = 0.0f;
    if (v < qv)
      x = __fmul_rn(q[(long long)(row0 + rl0 + v / nq) * q_ld + (long long)(g * nq + v % nq) * HD + d], scale);
    qs[v * KS + d] = x;
  }
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const float *Kg = kc + (long long)g * seq * HD, *Vg = vc + (long long)g * seq * HD;
  // Tile k into buffer k & 1: K row by row into the padded rows (a lane per row), V in one copy.
  auto issue = [&](int k) {
    const int t = k * kTile, cnt = min(kTile, vis_max - t), b = k & 1;
    if (lane == 0)
      mbar_arrive_expect_tx(&bar[b], 2u * cnt * HD * sizeof(float));
    __syncwarp();
    if (lane < cnt)
      bulk_g2s(Kb + (b * kTile + lane) * KS, Kg + (long long)(t + lane) * HD, HD * sizeof(float), &bar[b]);
    if (lane == 0)
      bulk_g2s(Vb + b * kTile * HD, Vg + (long long)t * HD, (unsigned)cnt * HD * sizeof(float), &bar[b]);
  };
  if (warp == 0)
    issue(0);
  auto out_of = [&](int v, int chunk) {  // partial of query v, chunk `chunk`
    return part + (((long long)(rl0 + v / nq) * n_heads + g * nq + v % nq) * cstride + chunk) * (HD + 2);
  };
  // Score / softmax role: queries 16 warp + lv + 4 i, positions lp + 8 j.
  const int lv = lane >> 3, lp = lane & 7, v0 = kQW * warp;
  int vis[kQL], len[kQL], cur[kQL];
  float mrun[kQL], lrun[kQL];
#pragma unroll
  for (int i = 0; i < kQL; i++) {
    cur[i] = -1, mrun[i] = -FLT_MAX, lrun[i] = 0.0f;
    const int v = v0 + lv + 4 * i, r = row0 + rl0 + v / nq;
    vis[i] = v < qv ? base + r + 1 : 0;
    len[i] = tile_plan(r, rblock, m, base, n_kv, limit, workers).len;
  }
  // P.V role: the warp's kQW queries x elements DL lane ...
  float acc[kQW][DL];
#pragma unroll
  for (int x = 0; x < kQW; x++)
#pragma unroll
    for (int e = 0; e < DL; e++)
      acc[x][e] = 0.0f;
  int failed = -1;  // the tile whose copy did not complete in time
  for (int k = 0; k < ntiles; k++) {
    const int t = k * kTile, cnt = min(kTile, vis_max - t), b = k & 1;
    if (!__syncthreads_and(mbar_wait_bounded(&bar[b], (k >> 1) & 1))) {
      failed = k;
      break;
    }
    if (warp == 0 && k + 1 < ntiles)
      issue(k + 1);  // its buffer's last readers finished before the barrier that ended the previous tile
    const float *Kt = Kb + b * kTile * KS;
    float s[kQL][4];
#pragma unroll
    for (int i = 0; i < kQL; i++)
#pragma unroll
      for (int j = 0; j < 4; j++)
        s[i][j] = 0.0f;
    float4 qq[kQL], kk[4];
#pragma unroll
    for (int i = 0; i < kQL; i++)
      qq[i] = *reinterpret_cast<const float4 *>(qs + (v0 + lv + 4 * i) * KS);
#pragma unroll
    for (int j = 0; j < 4; j++)
      kk[j] = *reinterpret_cast<const float4 *>(Kt + (lp + 8 * j) * KS);
#pragma unroll 2
    for (int d = 0; d < HD; d += 4) {
      // The next four elements' operands are read before this step's FMAs (the last step re-reads its own).
      const int dn = d + 4 < HD ? d + 4 : d;
      float4 qn[kQL], kn[4];
#pragma unroll
      for (int i = 0; i < kQL; i++)
        qn[i] = *reinterpret_cast<const float4 *>(qs + (v0 + lv + 4 * i) * KS + dn);
#pragma unroll
      for (int j = 0; j < 4; j++)
        kn[j] = *reinterpret_cast<const float4 *>(Kt + (lp + 8 * j) * KS + dn);
#pragma unroll
      for (int i = 0; i < kQL; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
          s[i][j] = __fmaf_rn(qq[i].x, kk[j].x, s[i][j]);
          s[i][j] = __fmaf_rn(qq[i].y, kk[j].y, s[i][j]);
          s[i][j] = __fmaf_rn(qq[i].z, kk[j].z, s[i][j]);
          s[i][j] = __fmaf_rn(qq[i].w, kk[j].w, s[i][j]);
        }
#pragma unroll
      for (int i = 0; i < kQL; i++)
        qq[i] = qn[i];
#pragma unroll
      for (int j = 0; j < 4; j++)
        kk[j] = kn[j];
    }
    // Online softmax, query by query. The 8 lanes of a query agree on whether it sees the tile, and every shuffle runs
    // in every lane; the state only moves where the query sees positions.
#pragma unroll
    for (int i = 0; i < kQL; i++) {
      const int v = v0 + lv + 4 * i, nv = max(0, min(kTile, vis[i] - t));
      const bool live = nv > 0;
      float alpha = 1.0f;
      int marker = -2;  // for P.V: -2 nothing, -1 first chunk, else the chunk to write out first
      if (live) {
        const int ck = t / len[i];
        if (ck != cur[i]) {
          if (cur[i] >= 0 && lp == 0) {
            float *o = out_of(v, cur[i]);
            o[HD] = mrun[i];
            o[HD + 1] = lrun[i];
          }
          marker = cur[i];
          cur[i] = ck;
          mrun[i] = -FLT_MAX, lrun[i] = 0.0f;
        }
      }
      float tmax = -FLT_MAX;
#pragma unroll
      for (int j = 0; j < 4; j++)
        if (lp + 8 * j < nv)
          tmax = fmaxf(tmax, s[i][j]);
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
      if (live && tmax > mrun[i]) {
        alpha = exp512_dev(__fsub_rn(mrun[i], tmax));
        lrun[i] = __fmul_rn(lrun[i], alpha);
        mrun[i] = tmax;
      }
      float e[4];
#pragma unroll
      for (int j = 0; j < 4; j++)
        e[j] = lp + 8 * j < nv ? exp512_dev(__fsub_rn(s[i][j], mrun[i])) : 0.0f;
      // Tile sum: lanes[p] = e[p] + e[16 + p] (p = lp: this lane's j = 0 and 2; p = 8 + lp: j = 1 and 3), t8[p] =
      // lanes[8 + p] + lanes[p] (this lane), t4[p] = t8[4 + p] + t8[p] (lanes lp and lp ^ 4), then
      // (t4[0] + t4[2]) + (t4[1] + t4[3]) (lanes lp ^ 2, then lp ^ 1): every lane of the query ends with the sum.
      float ts = __fadd_rn(__fadd_rn(e[1], e[3]), __fadd_rn(e[0], e[2]));
      ts = __fadd_rn(ts, __shfl_xor_sync(0xffffffffu, ts, 4));
      ts = __fadd_rn(ts, __shfl_xor_sync(0xffffffffu, ts, 2));
      ts = __fadd_rn(ts, __shfl_xor_sync(0xffffffffu, ts, 1));
      if (live)
        lrun[i] = __fadd_rn(lrun[i], ts);
#pragma unroll
      for (int j = 0; j < 4; j++)
        P[(lp + 8 * j) * kPStride + v] = e[j];
      if (lp == 0)
        al[v] = alpha, fl[v] = marker;
    }
    __syncwarp();
#pragma unroll
    for (int x = 0; x < kQW; x++) {
      const int v = v0 + x, f = fl[v];
      if (f >= 0) {  // the query's previous chunk is finished: write it out, start from zero
        float *o = out_of(v, f) + DL * lane;
#pragma unroll
        for (int e = 0; e < DL; e++) {
          o[e] = acc[x][e];
          acc[x][e] = 0.0f;
        }
      } else if (f == -1) {  // the query's first chunk starts here
#pragma unroll
        for (int e = 0; e < DL; e++)
          acc[x][e] = 0.0f;
      }
      const float a = al[v];
#pragma unroll
      for (int e = 0; e < DL; e++)
        acc[x][e] = __fmul_rn(acc[x][e], a);
    }
    const float *Vt = Vb + b * kTile * HD + DL * lane;
    const float *Pw = P + v0;
    // Row p's operands: the lane's DL elements of V and the warp's kQW probabilities (broadcasts).
    auto load_pv = [&](int p, float (&vv)[DL], float4 (&pe)[kQW / 4]) {
      if (DL == 4) {
        const float4 x4 = *reinterpret_cast<const float4 *>(Vt + p * HD);
        vv[0] = x4.x, vv[1 % DL] = x4.y, vv[2 % DL] = x4.z, vv[3 % DL] = x4.w;
      } else if (DL == 2) {
        const float2 x2 = *reinterpret_cast<const float2 *>(Vt + p * HD);
        vv[0] = x2.x, vv[1 % DL] = x2.y;
      } else {
        vv[0] = Vt[p * HD];
      }
#pragma unroll
      for (int y = 0; y < kQW / 4; y++)
        pe[y] = *reinterpret_cast<const float4 *>(Pw + p * kPStride + 4 * y);
    };
    float vv[DL];
    float4 pe[kQW / 4];
    load_pv(0, vv, pe);
#pragma unroll 2
    for (int p = 0; p < cnt; p++) {
      // The next row's operands are read before this row's FMAs (the last row re-reads its own).
      float vn[DL];
      float4 pn[kQW / 4];
      load_pv(p + 1 < cnt ? p + 1 : p, vn, pn);
#pragma unroll
      for (int y = 0; y < kQW / 4; y++) {
        const float ev[4] = {pe[y].x, pe[y].y, pe[y].z, pe[y].w};
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
          for (int e = 0; e < DL; e++)
            acc[4 * y + u][e] = __fmaf_rn(ev[u], vv[e], acc[4 * y + u][e]);
      }
#pragma unroll
      for (int e = 0; e < DL; e++)
        vv[e] = vn[e];
#pragma unroll
      for (int y = 0; y < kQW / 4; y++)
        pe[y] = pn[y];
    }
    __syncthreads();  // the buffers of this tile are refilled two tiles on (and P, al, fl by the next tile)
  }
  if (failed >= 0) {  // that tile's copy is the only one in flight: let it land (bounded) before leaving
    if (tid == 0)
      mbar_wait_bounded(&bar[failed & 1], (failed >> 1) & 1);
    return;
  }
  // The last chunk of every query.
#pragma unroll
  for (int i = 0; i < kQL; i++) {
    const int v = v0 + lv + 4 * i;
    if (lp == 0) {
      if (cur[i] >= 0) {
        float *o = out_of(v, cur[i]);
        o[HD] = mrun[i];
        o[HD + 1] = lrun[i];
      }
      fl[v] = cur[i];
    }
  }
  __syncwarp();
#pragma unroll
  for (int x = 0; x < kQW; x++) {
    const int v = v0 + x;
    if (v < qv && fl[v] >= 0) {
      float *o = out_of(v, fl[v]) + DL * lane;
#pragma unroll
      for (int e = 0; e < DL; e++)
        o[e] = acc[x][e];
    }
  }
}

// ---- host side ----------------------------------------------------------------------------------------------------

bool launched(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    kc_count_launch();
    return true;
  }
  return kc_fail("%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
}

int limit_for(int seq) { return (seq + kSplitMax - 1) / kSplitMax; }  // attention_max_chunks with a team of one

bool fast_shape(int n_heads, int n_kv, int hd) {
  const int nq = n_heads / n_kv;
  return (hd == 32 || hd == 64 || hd == 128) && nq <= kMaxNq && kMaxNq % nq == 0;
}

// Whether merge_warp_kernel can quantize a head's outputs in gs-groups: whole groups of hd / 32 elements per lane, a
// power-of-two number of lanes per group.
bool merge_warp_quantizes(int hd, int gs) {
  const int dl = hd / 32, lanes = gs / dl;
  return gs > 0 && hd % gs == 0 && gs % dl == 0 && lanes <= 32 && (lanes & (lanes - 1)) == 0;
}

// Shared-memory limits of the fast kernels, raised once per device.
bool smem_ready(int hd) {
  const void *split = hd == 128  ? reinterpret_cast<const void *>(split_kernel<128>)
                      : hd == 64 ? reinterpret_cast<const void *>(split_kernel<64>)
                                 : reinterpret_cast<const void *>(split_kernel<32>);
  const void *tiled = hd == 128  ? reinterpret_cast<const void *>(tiled_kernel<128>)
                      : hd == 64 ? reinterpret_cast<const void *>(tiled_kernel<64>)
                                 : reinterpret_cast<const void *>(tiled_kernel<32>);
  return kc_allow_smem(split, (int)split_smem_bytes(hd, kMaxNq)) == cudaSuccess &&
         kc_allow_smem(tiled, (int)tiled_smem_bytes(hd)) == cudaSuccess;
}

// Rows of the tiled variant's CTA: whole blocks of 16 / nq rows, 64 query vectors at most.
int tiled_rows_per_cta(int nq) {
  const int rb = tile_rblock(nq), blocks = kTQ / (rb * nq);
  return (blocks < 1 ? 1 : blocks) * rb;
}

// Rows of partials the work holds: the rows asked for, capped by a 512 MiB budget (longer batches run in waves),
// never less than one.
int work_rows(int n_heads, int head_dim, int seq_len, int rows) {
  const size_t per_row = (size_t)n_heads * limit_for(seq_len) * (head_dim + 2) * sizeof(float);
  const size_t fit = ((size_t)512 << 20) / per_row;
  return (int)(fit < 1 ? 1 : fit < (size_t)rows ? fit : (size_t)rows);
}

size_t partial_bytes(int n_heads, int head_dim, int seq_len, int rows) {
  return (size_t)work_rows(n_heads, head_dim, seq_len, rows) * n_heads * limit_for(seq_len) * (head_dim + 2) *
         sizeof(float);
}

unsigned *work_tickets(AttentionWork *w) { return reinterpret_cast<unsigned *>(w->partial + w->capacity); }

// One row (decode) or a batch of rows of attention into out (row stride out_ld), optionally quantized into oq/os.
bool attention_rows(const char *name, float *out, long long out_ld, int8_t *oq, float *os, const float *q,
                    long long q_ld, const float *kc, const float *vc, AttentionWork *w, int n_heads, int n_kv, int hd,
                    int seq, const int *pos_dev, int pos0, int rows, int gs, const RopeStep *rope = nullptr) {
  if (!w || !w->partial)
    return kc_fail("%s: attention work is not initialized", name);
  if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv || hd <= 0 || hd > kMaxHd || seq <= 0 || rows < 0 ||
      n_heads / n_kv > 1024)
    return kc_fail("%s: unsupported heads %d / KV heads %d / head_dim %d / context %d", name, n_heads, n_kv, hd, seq);
  if (n_heads != w->n_heads || hd != w->head_dim || limit_for(seq) > w->max_chunks)
    return kc_fail("%s: shape differs from the one the work was initialized for", name);
  if (oq && (gs <= 0 || (n_heads / n_kv * hd) % gs || out_ld % gs))
    return kc_fail("%s: group size %d does not divide a KV head's outputs", name, gs);
  if (!pos_dev && (pos0 < 0 || pos0 + rows > seq))
    return kc_fail("%s: positions %d..%d outside the context of %d", name, pos0, pos0 + rows - 1, seq);
  if (rows == 0)
    return true;
  const int nq = n_heads / n_kv, limit = w->max_chunks, workers = w->workers > 0 ? w->workers : 1;
  const bool fast = fast_shape(n_heads, n_kv, hd);
  if (fast && !smem_ready(hd))
    return kc_fail("%s: cannot reserve shared memory for the attention kernels", name);
  const bool fused_q = oq && hd % gs == 0;  // the merge quantizes whole groups inside a head
  const int slot = hd + 2, merge_threads = (hd + 31) / 32 * 32;
  cudaStream_t st = kc_stream();
  if (rows == 1) {
    bool merged = false;  // the split kernel merged the partials itself
    if ((size_t)n_heads * limit * slot > w->capacity)
      return kc_fail("%s: attention work too small", name);
    if (!fast) {
      kc_launch_pdl(split_generic_kernel, dim3(n_heads), dim3(limit), 0, st, q, kc, vc, pos_dev, pos0, n_heads, n_kv,
                    hd, seq, limit, workers, limit, w->partial);
    } else {
      void (*k)(const float *, const float *, const float *, const int *, int, int, int, int, int, int, int, float *,
                unsigned *, float *, int8_t *, float *, int, int, RopeStep) =
          hd == 128 ? split_kernel<128> : hd == 64 ? split_kernel<64> : split_kernel<32>;
      cudaLaunchConfig_t cfg = {};
      // About one wave of clusters (as many as fit at once): each walks the chunks y, y + gridDim.y, ... of the row.
      int clusters = 0;
      cfg.gridDim = dim3(n_kv, limit, kSplitCtas);
      cfg.blockDim = dim3(kSplitThreads);
      cfg.dynamicSmemBytes = split_smem_bytes(hd, nq);
      cfg.stream = st;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = kSplitCtas;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&clusters, k, &cfg) != cudaSuccess || clusters < 1) {
        cudaGetLastError();
        clusters = kc_device_sms() / kSplitCtas;
      }
      const int per_kv = clusters / n_kv;
      cfg.gridDim.y = per_kv < 1 ? 1 : per_kv < limit ? per_kv : limit;
      // The fused merge quantizes in the warp (merge_warp_quantizes); other group sizes merge in merge_kernel.
      unsigned *tickets =
          n_kv <= kSplitTickets && (!fused_q || merge_warp_quantizes(hd, gs)) ? work_tickets(w) : nullptr;
      if (tickets)
        merged = true;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = kc_pdl_enabled() ? 1 : 0;
      cfg.numAttrs = 2;
      // A position read from device memory is the decode step's: the cache rows below it may be read early.
      cudaLaunchKernelEx(&cfg, k, q, kc, vc, pos_dev, pos0, n_kv, nq, seq, limit, workers, limit, w->partial, tickets,
                         out, fused_q ? oq : (int8_t *)nullptr, fused_q ? os : (float *)nullptr, gs,
                         pos_dev ? 1 : 0, rope ? *rope : RopeStep{});
    }
    if (!launched(name))
      return false;
    if (!merged)
      kc_launch_pdl(merge_kernel, dim3(n_heads, 1), dim3(merge_threads), 0, st, out, out_ld,
                  fused_q ? oq : (int8_t *)nullptr, fused_q ? os : (float *)nullptr, (const float *)w->partial,
                    pos_dev, pos0, 0, 1, 0, n_heads, n_kv, hd, seq, limit, workers, limit, gs);
    if (!merged && !launched(name))
      return false;
  } else {
    // Waves of rows whose partials fit the work; the chunk stride is the most chunks a row of the wave can have.
    const int R = tiled_rows_per_cta(nq), rblock = tile_rblock(nq);
    for (int row0 = 0; row0 < rows;) {
      int wave = rows - row0, cstride = limit;
      for (;;) {
        if (!pos_dev) {
          cstride = 1;
          for (int r = row0; r < row0 + wave; r += rblock) {
            const int c = tile_plan(r, rblock, rows, pos0, n_kv, limit, workers).chunks;
            cstride = c > cstride ? c : cstride;
          }
          const int c = tile_plan(row0 + wave - 1, rblock, rows, pos0, n_kv, limit, workers).chunks;
          cstride = c > cstride ? c : cstride;
        }
        const size_t fit = w->capacity / ((size_t)n_heads * cstride * slot);
        if (fit >= (size_t)wave)
          break;
        if (fit < 1)
          return kc_fail("%s: attention work too small", name);
        wave = (int)fit;
      }
      if (!fast) {
        if (pos_dev)
          return kc_fail("%s: a batch at device positions needs head_dim 32, 64 or 128", name);
        kc_launch_pdl(tiled_generic_kernel, dim3(n_heads, wave), dim3(cstride), 0, st, q, q_ld, kc, vc, pos0, row0,
                      wave, rows, n_heads, n_kv, hd, seq, limit, workers, cstride, w->partial);
      } else {
        void (*k)(const float *, long long, const float *, const float *, const int *, int, int, int, int, int, int,
                  int, int, int, int, int, float *) =
            hd == 128 ? tiled_kernel<128> : hd == 64 ? tiled_kernel<64> : tiled_kernel<32>;
        kc_launch_pdl(k, dim3(n_kv, (wave + R - 1) / R), dim3(kTWarps * 32), tiled_smem_bytes(hd), st, q, q_ld, kc, vc,
                      pos_dev, pos0, row0, wave, rows, R, n_kv, nq, seq, limit, workers, cstride, w->partial);
      }
      if (!launched(name))
        return false;
      if (fast && (!fused_q || merge_warp_quantizes(hd, gs))) {
        void (*mk)(float *, long long, int8_t *, float *, const float *, const int *, int, int, int, int, int, int,
                   int, int, int, int, int) =
            hd == 128 ? merge_warp_kernel<128> : hd == 64 ? merge_warp_kernel<64> : merge_warp_kernel<32>;
        kc_launch_pdl(mk, dim3((unsigned)(((long long)wave * n_heads + 7) / 8)), dim3(256), 0, st, out, out_ld,
                      fused_q ? oq : (int8_t *)nullptr, fused_q ? os : (float *)nullptr, (const float *)w->partial,
                      pos_dev, pos0, row0, rows, wave, n_heads, n_kv, seq, limit, workers, cstride, gs);
      } else {
        kc_launch_pdl(merge_kernel, dim3(n_heads, wave), dim3(merge_threads), 0, st, out, out_ld,
                      fused_q ? oq : (int8_t *)nullptr, fused_q ? os : (float *)nullptr, (const float *)w->partial,
                      pos_dev, pos0, row0, rows, 1, n_heads, n_kv, hd, seq, limit, workers, cstride, gs);
      }
      if (!launched(name))
        return false;
      row0 += wave;
    }
  }
  if (oq && !fused_q) {
    if (kc_launch_quantize_rows(oq, os, out, out_ld, rows, n_heads * hd, gs, st) != 0)
      return kc_fail("%s: CUDA launch failed: %s", name, cudaGetErrorString(cudaGetLastError()));
    kc_count_launch();
  }
  return true;
}

// The merge tickets past the partials (kSplitTickets words, zeroed by k_attention_init_rows).
}  // namespace

extern "C" {

size_t k_attention_bytes_rows(int n_heads, int n_kv_heads, int head_dim, int seq_len, int rows) {
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || seq_len <= 0 || rows <= 0)
    return 0;
  return partial_bytes(n_heads, head_dim, seq_len, rows) + kSplitTickets * sizeof(unsigned);
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
  work->partial = reinterpret_cast<float *>(base);
  work->max_chunks = limit_for(seq_len);
  work->n_heads = n_heads;
  work->head_dim = head_dim;
  work->workers = 1;
  work->external = external;
  work->capacity = partial_bytes(n_heads, head_dim, seq_len, rows) / sizeof(float);
  if (cudaMemsetAsync(work_tickets(work), 0, kSplitTickets * sizeof(unsigned), kc_stream()) != cudaSuccess) {
    cudaGetLastError();
    if (!external)
      cudaFree(base);
    memset(work, 0, sizeof(*work));
    kc_fail("k_attention_init_rows: cannot clear the merge tickets");
  }
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

int k_rope_attention_q8_step_ok(int n_heads, int n_kv_heads, int head_dim, int gs) {
  return n_heads > 0 && n_kv_heads > 0 && n_heads % n_kv_heads == 0 && n_kv_heads <= kSplitTickets &&
         fast_shape(n_heads, n_kv_heads, head_dim) && (gs <= 0 || merge_warp_quantizes(head_dim, gs));
}

void k_rope_attention_q8_step(float *out, int8_t *oq, float *os, const float *q, const float *k, const float *v,
                              float *key_cache, float *value_cache, const float *table, AttentionWork *work,
                              int n_heads, int n_kv_heads, int head_dim, int seq_len, const int *position, int gs) {
  if (!position || !q || !k || !v || !table || !key_cache || !value_cache ||
      !k_rope_attention_q8_step_ok(n_heads, n_kv_heads, head_dim, oq ? gs : 0)) {
    kc_fail("k_rope_attention_q8_step: needs a device position, head_dim 32, 64 or 128, query heads per KV head "
            "dividing 16, and a group size whose groups a warp's lanes hold");
    return;
  }
  const long long ld = (long long)n_heads * head_dim;
  const RopeStep rope = {k, v, table, key_cache, value_cache};
  attention_rows("k_rope_attention_q8_step", out, ld, oq, os, q, ld, key_cache, value_cache, work, n_heads,
                 n_kv_heads, head_dim, seq_len, position, 0, 1, gs, &rope);
}

void k_attention_q8_rows(float *out, int8_t *oq, float *os, const float *q, const float *key_cache,
                         const float *value_cache, AttentionWork *work, int n_heads, int n_kv_heads, int head_dim,
                         int seq_len, const int *position, int pos0, int rows, int gs) {
  const long long ld = (long long)n_heads * head_dim;
  attention_rows("k_attention_q8_rows", out, ld, oq, os, q, ld, key_cache, value_cache, work, n_heads, n_kv_heads,
                 head_dim, seq_len, position, pos0, rows, gs);
}

}  // extern "C"
