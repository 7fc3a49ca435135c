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

constexpr int kThreads = 256;
constexpr int kTile = 32;        // positions per tile of the batched variant (its TILED_POS)
constexpr int kSplitMax = 256;   // positions of a split chunk at most (attention_chunks' shortest bound)
constexpr int kQV = 64;          // query vectors of a batched CTA
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
// [k n / 4, (k + 1) n / 4) of the chunk's n <= 256 positions (one bulk copy) and computes their scores for the group's
// nq heads, which it stores into every CTA of the cluster (distributed shared memory); after a cluster barrier each
// CTA holds all the chunk's scores, takes the maximum, exp512 and the 16-lane exp-sum per head (the same in every
// CTA), and runs the P.V chains of its quarter of the head's elements over V[chunk rows][its quarter] (cp.async
// copies). So each K and V element is read once. A cluster walks chunks y, y + gridDim.y, ... (about one wave of
// clusters). With `tickets`, the CTA that finishes a KV head's last chunk also merges the group's partials (the
// arithmetic of merge_kernel) and writes its outputs, so no second launch waits on the partials.
constexpr int kSplitCtas = 4;
constexpr int kSplitThreads = 256;
constexpr int kSplitTickets = 256;  // KV heads the fused merge serves (a ticket word each, past the partials)

// Floats before the mbarrier: K quarter [kSplitMax / 4][hd], V quarter [kSplitMax][hd / 4], Q [nq][hd],
// scores [nq][kSplitMax], the per-head maximum and exp-sum.
__host__ __device__ constexpr size_t split_smem_floats(int hd, int nq) {
  return (size_t)(kSplitMax / kSplitCtas) * hd + (size_t)kSplitMax * (hd / kSplitCtas) + (size_t)nq * hd +
         (size_t)nq * kSplitMax + 2 * kMaxNq;
}
__host__ __device__ constexpr size_t split_smem_bytes(int hd, int nq) {
  return split_smem_floats(hd, nq) * sizeof(float) + sizeof(uint64_t);
}

__device__ __forceinline__ void st_cluster_f32(float *local, unsigned rank, float v) {
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

__device__ __forceinline__ void st_cluster_u32(unsigned *local, unsigned rank, unsigned v) {
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(remote), "r"(v) : "memory");
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
// for the nq heads at once, chunk partials staged in shared memory a block at a time.
template <int HD>
__device__ void merge_group(float *sm, int sm_floats, const float *part, int g, int nq, int chunks, int cstride,
                            float *out, int8_t *oq, float *os, int gs) {
  constexpr int slot = HD + 2, nt = kSplitThreads, kOut = (kMaxNq * HD + nt - 1) / nt;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, outs = nq * HD;
  float *mxs = sm, *vals = mxs + kMaxNq, *scl = vals + nq * HD, *wts = scl + nq * HD;
  // At least 8 chunks a block for every shape fast_shape admits (the K and V quarters alone hold 128 hd floats).
  const int cb = (sm_floats - (kMaxNq + 2 * nq * HD)) / (nq * (slot + 1));
  float *stage = wts + nq * cb;
  const float *pg = part + (long long)g * nq * cstride * slot;
  for (int hh = warp; hh < nq; hh += nt / 32) {
    float mx = -FLT_MAX;
    for (int c = lane; c < chunks; c += 32)
      mx = fmaxf(mx, __ldcg(pg + ((long long)hh * cstride + c) * slot + HD));
#pragma unroll
    for (int off = 16; off; off >>= 1)
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0)
      mxs[hh] = mx;
  }
  float sum[kOut], acc[kOut];
#pragma unroll
  for (int u = 0; u < kOut; u++)
    sum[u] = 0.0f, acc[u] = 0.0f;
  for (int c0 = 0; c0 < chunks; c0 += cb) {
    const int nc = chunks - c0 < cb ? chunks - c0 : cb;
    __syncthreads();  // the maxima are in; the previous block's reads are done
    for (int i = tid; i < nq * nc * slot; i += nt) {
      const int hh = i / (nc * slot), rem = i - hh * nc * slot;
      stage[i] = __ldcg(pg + ((long long)hh * cstride + c0) * slot + rem);
    }
    __syncthreads();
    for (int i = tid; i < nq * nc; i += nt) {
      const int hh = i / nc;
      wts[i] = expf_libc(__fsub_rn(stage[i * slot + HD], mxs[hh]));
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kOut; u++) {
      const int o = tid + u * nt;
      if (o < outs) {
        const int hh = o / HD, d = o - hh * HD;
        const float *sp = stage + hh * nc * slot, *wp = wts + hh * nc;
        for (int c = 0; c < nc; c++) {
          const float w = wp[c];
          sum[u] = __fadd_rn(sum[u], __fmul_rn(w, sp[c * slot + HD + 1]));
          acc[u] = __fadd_rn(acc[u], __fmul_rn(w, sp[c * slot + d]));
        }
      }
    }
  }
  float *dst = out + (long long)g * outs;
  int bad = 0;
#pragma unroll
  for (int u = 0; u < kOut; u++) {
    const int o = tid + u * nt;
    if (o < outs) {
      const float v = __fdiv_rn(acc[u], sum[u]);
      dst[o] = v;
      vals[o] = v;
      bad |= !isfinite(v);
    }
  }
  if (!oq || gs <= 0 || HD % gs)
    return;
  if (__syncthreads_or(bad)) {
    if (tid == 0)
      kc_raise(KC_ERR_NONFINITE);
    return;
  }
  // Group maxima of |v| (order-free), a warp per group; scale = max / 127.
  for (int grp = warp; grp < outs / gs; grp += nt / 32) {
    float a = 0.0f;
    for (int i = lane; i < gs; i += 32)
      a = fmaxf(a, fabsf(vals[grp * gs + i]));
#pragma unroll
    for (int off = 16; off; off >>= 1)
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
    if (lane == 0)
      scl[grp] = __fdiv_rn(a, 127.0f);
  }
  __syncthreads();
  const long long e0 = (long long)g * outs;
  for (int o = tid; o < outs; o += nt) {
    const float sc = scl[o / gs];
    oq[e0 + o] = (int8_t)quantize_value(vals[o], sc);
    if (o % gs == 0)
      os[(e0 + o) / gs] = sc;
  }
}

template <int HD>
__global__ void __launch_bounds__(kSplitThreads, 3) split_kernel(const float *q, const float *kc, const float *vc,
                                                              const int *pos_dev, int pos0, int n_kv, int nq, int seq,
                                                              int limit, int workers, int cstride, float *part,
                                                              unsigned *tickets, float *out, int8_t *oq, float *os,
                                                              int gs) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int QD = HD / kSplitCtas;  // elements of the head this CTA's P.V covers
  extern __shared__ __align__(16) float sm[];
  const int sm_floats = (int)split_smem_floats(HD, nq);
  float *Kq = sm, *Vq = Kq + (kSplitMax / kSplitCtas) * HD, *Q = Vq + kSplitMax * QD, *S = Q + nq * HD;
  float *hmax = S + nq * kSplitMax, *hsum = hmax + kMaxNq;
  uint64_t *bar = reinterpret_cast<uint64_t *>(sm + sm_floats);
  __shared__ unsigned fails[kSplitCtas];
  __shared__ int last;
  static_assert(kSplitCtas == 4, "the failure vote reads four slots");
  const int g = blockIdx.x, k = blockIdx.z, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
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
  for (int i = tid; i < nq * HD; i += kSplitThreads)
    Q[i] = q[(long long)g * nq * HD + i];
  __syncthreads();
  // The cluster walks chunks blockIdx.y, blockIdx.y + gridDim.y, ...; every CTA of it takes the same steps.
  unsigned phase = 0;
  for (int c = blockIdx.y; c < chunks; c += gridDim.y) {
    const int t0 = (int)((long long)P * c / chunks), n = (int)((long long)P * (c + 1) / chunks) - t0;  // <= 256
    const int k0 = n * k / kSplitCtas, kn = n * (k + 1) / kSplitCtas - k0;  // this CTA's K rows
    const float *Kg = kc + ((long long)g * seq + t0) * HD, *Vg = vc + ((long long)g * seq + t0) * HD;
    if (tid == 0 && kn > 0) {
      mbar_arrive_expect_tx(bar, (unsigned)kn * HD * sizeof(float));
      bulk_g2s(Kq, Kg + (long long)k0 * HD, (unsigned)kn * HD * sizeof(float), bar);
    }
    // V[chunk rows][k QD .. (k + 1) QD): QD / 4 16-byte pieces a row.
    for (int i = tid; i < n * (QD / 4); i += kSplitThreads) {
      const int t = i / (QD / 4), p4 = i - t * (QD / 4);
      cp_async16(Vq + t * QD + 4 * p4, Vg + (long long)t * HD + k * QD + 4 * p4);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    bool ok = true;
    if (kn > 0) {
      ok = __syncthreads_and(mbar_wait_bounded(bar, phase));
      phase ^= 1u;
    }
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
      break;  // the whole cluster stops in the same iteration (the error is raised)
    }
    // Per head (a warp each): the maximum, exp512 in place, the exp-sum in 16 lanes then the tree.
    for (int h = warp; h < nq; h += kSplitThreads / 32) {
      float *sh = S + h * kSplitMax;
      float mx = -FLT_MAX;
      for (int t = lane; t < n; t += 32)
        mx = fmaxf(mx, sh[t]);
#pragma unroll
      for (int off = 16; off; off >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      for (int t = lane; t < n; t += 32)
        sh[t] = exp512_dev(__fsub_rn(sh[t], mx));
      __syncwarp();
      float vs = 0.0f;
      if (lane < 16)
        for (int t = lane; t < n; t += 16)
          vs = __fadd_rn(vs, sh[t]);
      vs = tree16_lanes(vs);
      if (lane == 0)
        hmax[h] = mx, hsum[h] = vs;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // P.V: a chain per (head, element of this CTA's quarter) over the chunk's positions in order.
    for (int i = tid; i < nq * QD; i += kSplitThreads) {
      const int h = i / QD, d = i - h * QD;
      const float *e = S + h * kSplitMax;
      float acc = 0.0f;
      int t = 0;
      for (; t + 8 <= n; t += 8) {
        float ev[8], vv[8];
#pragma unroll
        for (int u = 0; u < 8; u++)
          ev[u] = e[t + u], vv[u] = Vq[(t + u) * QD + d];
#pragma unroll
        for (int u = 0; u < 8; u++)
          acc = __fmaf_rn(ev[u], vv[u], acc);
      }
      for (; t < n; t++)
        acc = __fmaf_rn(e[t], Vq[t * QD + d], acc);
      part[((long long)(g * nq + h) * cstride + c) * (HD + 2) + k * QD + d] = acc;
    }
    if (k == 0 && tid < nq) {
      float *o = part + ((long long)(g * nq + tid) * cstride + c) * (HD + 2);
      o[HD] = hmax[tid];
      o[HD + 1] = hsum[tid];
    }
    // The scores, K and V buffers are refilled by the cluster's next chunk: every CTA is done with them first.
    cluster_sync_all();
  }
  if (!tickets)
    return;
  // Every CTA that took chunks counts them (after a failure too, so the count stays whole); the one that completes
  // the KV head's 4 x chunks merges it and resets the ticket for the next call.
  const unsigned mine = (unsigned)((chunks - 1 - (int)blockIdx.y) / (int)gridDim.y + 1);
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned before = atomicAdd(tickets + g, mine);
    last = before + mine == (unsigned)(kSplitCtas * chunks);
    if (last) {
      tickets[g] = 0u;
      __threadfence();
    }
  }
  __syncthreads();
  if (last)
    merge_group<HD>(sm, sm_floats, part, g, nq, chunks, cstride, out, oq, os, gs);
}

// ---- the tiled variant for a batch of rows (prefill) ---------------------------------------------------------------
// CTA (KV head g, group of R rows = whole or part blocks): its query vectors v = (row - first row) * nq + head, at
// most 64, over the 32-position tiles of the group's causal range. Per tile: K and V rows by bulk copy (two buffers,
// the next tile's copy in flight), K transposed for the score tiles; then each thread takes 2 queries x 4 positions:
// their scores (chains over the head's elements in order) and, with the 8 threads that share the queries (8
// consecutive lanes, 32 positions), the online softmax of the tile: the tile maximum by shuffles, the rescale of the
// running sum, exp512, and the tile sum in the reference's order (positions j and 16 + j, then the 16-lane tree) by
// shuffles across the 8 lanes. Every lane of a group keeps the queries' running maximum, sum and chunk. Then P.V
// (4 queries x hd/16 elements a thread, chains over the tile's positions in order). A query whose chunk (its block's
// plan) changes at a tile writes the finished chunk's partial first and starts again from zero.
__host__ __device__ constexpr size_t tiled_smem_bytes(int hd) {
  return ((size_t)4 * kTile * hd + (size_t)hd * kTile + (size_t)hd * kQV + (size_t)kTile * kQV + 2 * kQV) *
             sizeof(float) + 2 * sizeof(uint64_t);
}

template <int HD>
__global__ void __launch_bounds__(kThreads) tiled_kernel(const float *q, long long q_ld, const float *kc,
                                                         const float *vc, const int *pos_dev, int pos0, int row0,
                                                         int rows, int m, int R, int n_kv, int nq, int seq, int limit,
                                                         int workers, int cstride, float *part) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) float sm[];
  float *Kb = sm, *Vb = Kb + 2 * kTile * HD, *kt = Vb + 2 * kTile * HD, *qs = kt + HD * kTile;
  float *P = qs + HD * kQV, *al = P + kTile * kQV;
  int *fl = reinterpret_cast<int *>(al + kQV);
  uint64_t *bar = reinterpret_cast<uint64_t *>(fl + kQV);
  constexpr int DB = HD / 16;
  const int g = blockIdx.x, tid = threadIdx.x;
  const int base = pos_dev ? *pos_dev : pos0;
  const int rl0 = blockIdx.y * R, nr = min(R, rows - rl0);  // rows of this CTA, from wave row rl0
  if (nr <= 0 || base < 0 || base + row0 + rl0 + nr > seq)
    return;  // the merge kernel reports bad positions
  const int qv = nr * nq, rblock = tile_rblock(nq), n_heads = n_kv * nq;
  const int vis_max = base + row0 + rl0 + nr, ntiles = (vis_max + kTile - 1) / kTile;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  // Queries, scaled, transposed: qs[d][v].
  for (int i = tid; i < kQV * HD; i += kThreads) {
    const int v = i / HD, d = i - v * HD;
    float x = 0.0f;
    if (v < qv)
      x = __fmul_rn(q[(long long)(row0 + rl0 + v / nq) * q_ld + (long long)(g * nq + v % nq) * HD + d], scale);
    qs[d * kQV + v] = x;
  }
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const float *Kg = kc + (long long)g * seq * HD, *Vg = vc + (long long)g * seq * HD;
  auto issue = [&](int k) {
    const int t = k * kTile, cnt = min(kTile, vis_max - t);
    const unsigned bytes = (unsigned)cnt * HD * sizeof(float);
    mbar_arrive_expect_tx(&bar[k & 1], 2 * bytes);
    bulk_g2s(Kb + (k & 1) * kTile * HD, Kg + (long long)t * HD, bytes, &bar[k & 1]);
    bulk_g2s(Vb + (k & 1) * kTile * HD, Vg + (long long)t * HD, bytes, &bar[k & 1]);
  };
  if (tid == 0)
    issue(0);
  auto out_of = [&](int v, int chunk) {  // partial of query v, chunk `chunk`
    return part + (((long long)(rl0 + v / nq) * n_heads + g * nq + v % nq) * cstride + chunk) * (HD + 2);
  };
  // Score / softmax role: queries 2 qp + i (i = 0, 1), positions 4 pq + j (j = 0..3) of each tile.
  const int qp = tid >> 3, pq = tid & 7;
  int vis[2], len[2], cur[2] = {-1, -1};
  float mrun[2] = {-FLT_MAX, -FLT_MAX}, lrun[2] = {0.0f, 0.0f};
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int v = 2 * qp + i, r = row0 + rl0 + v / nq;
    vis[i] = v < qv ? base + r + 1 : 0;
    len[i] = tile_plan(r, rblock, m, base, n_kv, limit, workers).len;
  }
  // P.V role: queries 4 qq.., elements DB dg...
  const int qq = tid >> 4, dg = tid & 15;
  float acc[4][DB];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int d = 0; d < DB; d++)
      acc[i][d] = 0.0f;
  int failed = -1;  // the tile whose copy did not complete in time
  for (int k = 0; k < ntiles; k++) {
    const int t = k * kTile, cnt = min(kTile, vis_max - t), b = k & 1;
    if (!__syncthreads_and(mbar_wait_bounded(&bar[b], (k >> 1) & 1))) {
      failed = k;
      break;
    }
    if (tid == 0 && k + 1 < ntiles)
      issue(k + 1);  // its buffer's last readers finished before the barrier above
    for (int i = tid; i < kTile * HD; i += kThreads) {
      const int p = i / HD, d = i - p * HD;
      kt[d * kTile + p] = p < cnt ? Kb[b * kTile * HD + i] : 0.0f;
    }
    __syncthreads();
    float s[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
#pragma unroll 8
    for (int d = 0; d < HD; d++) {
      const float2 qv2 = *reinterpret_cast<const float2 *>(qs + d * kQV + 2 * qp);
      const float4 kv4 = *reinterpret_cast<const float4 *>(kt + d * kTile + 4 * pq);
      s[0][0] = __fmaf_rn(qv2.x, kv4.x, s[0][0]);
      s[0][1] = __fmaf_rn(qv2.x, kv4.y, s[0][1]);
      s[0][2] = __fmaf_rn(qv2.x, kv4.z, s[0][2]);
      s[0][3] = __fmaf_rn(qv2.x, kv4.w, s[0][3]);
      s[1][0] = __fmaf_rn(qv2.y, kv4.x, s[1][0]);
      s[1][1] = __fmaf_rn(qv2.y, kv4.y, s[1][1]);
      s[1][2] = __fmaf_rn(qv2.y, kv4.z, s[1][2]);
      s[1][3] = __fmaf_rn(qv2.y, kv4.w, s[1][3]);
    }
    // Online softmax. The 4 groups of a warp may differ in whether they see the tile, so every shuffle runs in every
    // lane; the state only moves where the group sees positions.
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int v = 2 * qp + i, nv = max(0, min(kTile, vis[i] - t));
      const bool live = nv > 0;  // the same in all 8 lanes of the group
      float alpha = 1.0f;
      int marker = -2;  // for the P.V threads: -2 nothing, -1 first chunk, else the chunk to write out first
      if (live) {
        const int ck = t / len[i];
        if (ck != cur[i]) {
          if (cur[i] >= 0 && pq == 0) {
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
        if (4 * pq + j < nv)
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
        e[j] = 4 * pq + j < nv ? exp512_dev(__fsub_rn(s[i][j], mrun[i])) : 0.0f;
      // Tile sum: pair[p] = e[p] + e[16 + p] (p < 16: lanes pq < 4 hold p, pq + 4 hold 16 + p), t8[p] =
      // pair[8 + p] + pair[p] (p < 8: lanes pq and pq + 2), t4[p] = t8[4 + p] + t8[p] (lanes 0 and 1), then
      // (t4[0] + t4[2]) + (t4[1] + t4[3]) in lane 0 of the group.
      float a[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        a[j] = __fadd_rn(e[j], __shfl_xor_sync(0xffffffffu, e[j], 4));
        a[j] = __fadd_rn(a[j], __shfl_xor_sync(0xffffffffu, a[j], 2));
        a[j] = __fadd_rn(a[j], __shfl_xor_sync(0xffffffffu, a[j], 1));
      }
      const float tsum = __shfl_sync(0xffffffffu, __fadd_rn(__fadd_rn(a[0], a[2]), __fadd_rn(a[1], a[3])), 0, 8);
      if (live)
        lrun[i] = __fadd_rn(lrun[i], tsum);
#pragma unroll
      for (int j = 0; j < 4; j++)
        P[(4 * pq + j) * kQV + v] = e[j];
      if (pq == 0)
        al[v] = alpha, fl[v] = marker;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int v = 4 * qq + i, f = fl[v];
      if (f >= 0) {  // the query's previous chunk is finished: write it out, start from zero
        float *o = out_of(v, f);
#pragma unroll
        for (int d = 0; d < DB; d++) {
          o[dg * DB + d] = acc[i][d];
          acc[i][d] = 0.0f;
        }
      } else if (f == -1) {  // the query's first chunk starts here
#pragma unroll
        for (int d = 0; d < DB; d++)
          acc[i][d] = 0.0f;
      }
      const float a = al[v];
#pragma unroll
      for (int d = 0; d < DB; d++)
        acc[i][d] = __fmul_rn(acc[i][d], a);
    }
    const float *Vt = Vb + b * kTile * HD;
#pragma unroll 4
    for (int p = 0; p < cnt; p++) {
      const float4 pv = *reinterpret_cast<const float4 *>(P + p * kQV + 4 * qq);
      float vv[DB];
#pragma unroll
      for (int d = 0; d < DB; d += 4) {
        const float4 x = *reinterpret_cast<const float4 *>(Vt + p * HD + dg * DB + d);
        vv[d] = x.x, vv[d + 1] = x.y, vv[d + 2] = x.z, vv[d + 3] = x.w;
      }
      const float pr[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int d = 0; d < DB; d++)
          acc[i][d] = __fmaf_rn(pr[i], vv[d], acc[i][d]);
    }
    __syncthreads();  // the buffers of this tile are refilled two tiles on
  }
  if (failed >= 0) {  // that tile's copy is the only one in flight: let it land (bounded) before leaving
    if (tid == 0)
      mbar_wait_bounded(&bar[failed & 1], (failed >> 1) & 1);
    return;
  }
  // The last chunk of every query.
#pragma unroll
  for (int i = 0; i < 2; i++)
    if (pq == 0 && cur[i] >= 0) {
      float *o = out_of(2 * qp + i, cur[i]);
      o[HD] = mrun[i];
      o[HD + 1] = lrun[i];
    }
  __syncthreads();  // fl: the P.V threads read the final chunk of their queries from the score threads' state below
  if (pq == 0) {
    fl[2 * qp] = cur[0];
    fl[2 * qp + 1] = cur[1];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int v = 4 * qq + i;
    if (v < qv && fl[v] >= 0) {
      float *o = out_of(v, fl[v]);
#pragma unroll
      for (int d = 0; d < DB; d++)
        o[dg * DB + d] = acc[i][d];
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
  const int rb = tile_rblock(nq), blocks = kQV / (rb * nq);
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
                    int seq, const int *pos_dev, int pos0, int rows, int gs) {
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
                unsigned *, float *, int8_t *, float *, int) =
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
      unsigned *tickets = n_kv <= kSplitTickets ? work_tickets(w) : nullptr;
      if (tickets)
        merged = true;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = kc_pdl_enabled() ? 1 : 0;
      cfg.numAttrs = 2;
      cudaLaunchKernelEx(&cfg, k, q, kc, vc, pos_dev, pos0, n_kv, nq, seq, limit, workers, limit, w->partial, tickets,
                         out, fused_q ? oq : (int8_t *)nullptr, fused_q ? os : (float *)nullptr, gs);
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
        kc_launch_pdl(k, dim3(n_kv, (wave + R - 1) / R), dim3(kThreads), tiled_smem_bytes(hd), st, q, q_ld, kc, vc,
                      pos_dev, pos0, row0, wave, rows, R, n_kv, nq, seq, limit, workers, cstride, w->partial);
      }
      if (!launched(name))
        return false;
      kc_launch_pdl(merge_kernel, dim3(n_heads, wave), dim3(merge_threads), 0, st, out, out_ld,
                    fused_q ? oq : (int8_t *)nullptr, fused_q ? os : (float *)nullptr, (const float *)w->partial,
                    pos_dev, pos0, row0, rows, 1, n_heads, n_kv, hd, seq, limit, workers, cstride, gs);
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

void k_attention_q8_rows(float *out, int8_t *oq, float *os, const float *q, const float *key_cache,
                         const float *value_cache, AttentionWork *work, int n_heads, int n_kv_heads, int head_dim,
                         int seq_len, const int *position, int pos0, int rows, int gs) {
  const long long ld = (long long)n_heads * head_dim;
  attention_rows("k_attention_q8_rows", out, ld, oq, os, q, ld, key_cache, value_cache, work, n_heads, n_kv_heads,
                 head_dim, seq_len, position, pos0, rows, gs);
}

}  // extern "C"
