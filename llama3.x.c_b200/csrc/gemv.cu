// Q8_0 W8A8 decode GEMV for sm_100a: y[r] = sum over groups g of (float)dot_g(xq, wq[r]) * xs[g] * ws[r][g] with the
// epilogues of the reference's GEMV drivers (src/gemv.c:441-528: STORE / ADD / PARTIAL over 1-3 segments, SWIGLU on
// a w1/w3 pair).
//
// Arithmetic: every group dot is the exact int32 sum of gs int8 products (dp4a), and each output row accumulates
//   acc = fmaf((float)dot_g * xs[g], ws[r][g], acc)      for g = 0, 1, ..., ascending, from acc = 0
// which is the AMX-INT8 backend's rescale (amx_q8_chunk, src/gemm.c:604-608). The result is therefore bitwise the
// reference's AMX path and the tensor-core prefill GEMM of this library, and agrees with the reference's scalar and
// AVX-512 GEMVs within the reference's own Q8 budget (tests/kernels.c:138-170).
//
// Data movement: the weight bytes are HBM-bound. Each CTA owns a contiguous range of output rows (the static split of
// q8_team_static, src/gemv.c:483-490), walks it in sub-tiles of 32 physical weight rows that never straddle a
// segment, and streams each sub-tile through shared memory in 1 KiB K-chunks with TMA tensor copies: one 3-D box
// [8 K-blocks x 32 rows x 128 B] (128-byte swizzled; two 16-row halves from w1 and w3 for SwiGLU) for the weights and
// one box of the chunk's weight scales, completing on one mbarrier, several stages deep (TMA issue costs tens of
// cycles per instruction, so a stage is one or two instructions, not one per row or per 128 B). Inside a stage, lane r of every
// dot warp owns weight row r and warp w takes groups w, w+8, ... of the chunk, so the int32 dots need no shuffles and,
// thanks to the swizzle, 8 consecutive lanes read 8 distinct bank quads. A ninth warp runs the ordered fp32 chain for
// all 32 rows (one lane per row) from a double-buffered transposed buffer, writes the outputs and refills the freed
// stage. Dot warps and the chain warp hand the buffers over with named barriers; no CTA-wide barrier sits in the loop.
//
// Launch overlap: the kernel lets its dependent start at once (griddepcontrol.launch_dependents) and issues its first
// weight stage before waiting on the kernel it depends on (griddepcontrol.wait), so under programmatic dependent
// launch the weight stream overlaps the previous kernel's tail. Activations and outputs are touched only after the
// wait.
#include <cuda.h>
#include <string.h>

#include "common.cuh"
#include "kernels_cuda_internal.h"
#include "tmap.h"

namespace {

constexpr int kDotWarps = 8;
constexpr int kThreads = (kDotWarps + 1) * 32;  // 8 dot warps + 1 chain/producer warp
constexpr int kTileRows = 32;                   // physical weight rows per sub-tile (one per lane)
#ifndef KC_GEMV_CHUNK
#define KC_GEMV_CHUNK 1024
#endif
constexpr int kChunk = KC_GEMV_CHUNK;           // K bytes per stage
constexpr int kBoxCols = 128;                   // bytes per 128B-swizzled box row
constexpr int kBoxes = kChunk / kBoxCols;
constexpr int kWeightStage = kTileRows * kChunk;
constexpr int kFastGroups = kChunk / 64;            // groups of a full chunk at gs 64
constexpr int kWarpGroups = kFastGroups / kDotWarps;  // ... of them per dot warp
// Named barriers (0 is __syncthreads): T_FULL + b / T_EMPTY + b for the two chain buffers b.
#ifndef KC_GEMV_TBUF
#define KC_GEMV_TBUF 2
#endif
constexpr int kTBuf = KC_GEMV_TBUF;  // chain buffers: how many stages the dot warps may run ahead of the chain warp
constexpr int kBarTFull = 1, kBarTEmpty = 1 + kTBuf;
static_assert(kTBuf >= 2 && kTBuf <= 4, "chain buffers");

struct GemvSegDev {
  float *out;
  int d;
  int unit0;
};

// Tensor maps stay in parameter space (the TMA unit reads them there); the scalars travel in a separate by-value
// struct that the kernel copies into registers with static indices (dynamic indexing into parameter space turns
// every access into a slow generic load).
struct __align__(64) GemvMaps {
  CUtensorMap wmap[3];  // weights of each segment (w1 for SwiGLU), boxes [128 B x box_rows]
  CUtensorMap smap[3];  // weight scales, boxes [gpc floats x box_rows]
  CUtensorMap w3map;    // SwiGLU: w3 and its scales
  CUtensorMap s3map;
};

// Activation modes: the int8 values and scales as given, or fp32 values quantized (and first RMS-normalized) by every
// CTA into its shared memory.
enum { kActQ8 = 0, kActQuantize = 1, kActNormQuantize = 2 };

struct GemvArgs {
  GemvSegDev seg[3];
  int nseg;
  const int8_t *xq;
  const float *xs;
  const float *xf;     // kActQuantize / kActNormQuantize: fp32 activations
  const float *normw;  // kActNormQuantize: RMSNorm weights
  float eps;
  int act;
  KcGemvTail tail;     // work the last CTA to finish does once (kind 0: none)
  int n;        // inputs (K)
  int gs;
  int kind;     // KC_STORE / KC_ADD / KC_PARTIAL / KC_SWIGLU / KC_REDUCE_ADD
  int units;    // output rows over all segments
  int nchunks;
  int depth;    // pipeline stages
  int stage_bytes;
  int kblock;   // weight maps are 3-D k-block maps: one TMA instruction per stage (and per w1/w3 half)
  KcPeerGemv peer;  // KC_REDUCE_ADD: the ranks' slots and this rank's call counters
};

struct Sub {
  int seg, row0, cnt, unit;  // segment, its first local row, rows (units) in the sub-tile, global unit of row0
};

// The CTA's share of each segment, [lo, hi) in global units, and its sub-tile counts, kept in registers.
struct Plan {
  int lo[3], hi[3], nsub[3], unit0[3];
  int tile_shift;  // log2 of the sub-tile size (32 or 16 units)
};

__device__ __forceinline__ Plan make_plan(const GemvArgs &a, int u0, int u1, int tile_shift) {
  Plan p;
  p.tile_shift = tile_shift;
#pragma unroll
  for (int s = 0; s < 3; s++) {
    p.unit0[s] = a.seg[s].unit0;
    p.lo[s] = max(u0, a.seg[s].unit0);
    p.hi[s] = s < a.nseg ? min(u1, a.seg[s].unit0 + a.seg[s].d) : p.lo[s];
    p.nsub[s] = p.hi[s] > p.lo[s] ? ((p.hi[s] - p.lo[s] + (1 << tile_shift) - 1) >> tile_shift) : 0;
  }
  return p;
}

// Sub-tile k of the CTA's unit range: tiles of up to 2^tile_shift units that never cross a segment boundary.
__device__ __forceinline__ Sub subtile(const Plan &p, int k) {
  Sub r = {0, 0, 0, 0};
  int s = 0;
  if (k >= p.nsub[0]) {
    k -= p.nsub[0];
    s = 1;
    if (k >= p.nsub[1]) {
      k -= p.nsub[1];
      s = 2;
    }
  }
  const int lo = s == 0 ? p.lo[0] : s == 1 ? p.lo[1] : p.lo[2];
  const int hi = s == 0 ? p.hi[0] : s == 1 ? p.hi[1] : p.hi[2];
  const int u0s = s == 0 ? p.unit0[0] : s == 1 ? p.unit0[1] : p.unit0[2];
  r.seg = s;
  r.unit = lo + (k << p.tile_shift);
  r.row0 = r.unit - u0s;
  r.cnt = min(1 << p.tile_shift, hi - r.unit);
  return r;
}

__device__ __forceinline__ bool lane_active(bool swiglu, int lane, int cnt) {
  return swiglu ? (lane & 15) < cnt : lane < cnt;
}

// Named barriers with immediate ids: a register id makes ptxas reserve all 16 of the CTA's barriers, and the SM's
// barrier pool then holds one CTA of this kernel at a time.
template <int ID>
__device__ __forceinline__ void bar_sync_id() {
  asm volatile("bar.sync %0, %1;" ::"n"(ID), "n"(kThreads) : "memory");
}
template <int ID>
__device__ __forceinline__ void bar_arrive_id() {
  asm volatile("bar.arrive %0, %1;" ::"n"(ID), "n"(kThreads) : "memory");
}
// Barrier BASE + idx (idx < kTBuf), with the id an immediate in every branch.
template <int BASE>
__device__ __forceinline__ void bar_sync_named(int idx) {
  switch (idx) {
    case 0: bar_sync_id<BASE>(); break;
    case 1: bar_sync_id<BASE + 1>(); break;
    case 2: if (kTBuf > 2) bar_sync_id<BASE + (kTBuf > 2 ? 2 : 0)>(); break;
    default: if (kTBuf > 3) bar_sync_id<BASE + (kTBuf > 3 ? 3 : 0)>(); break;
  }
}
template <int BASE>
__device__ __forceinline__ void bar_arrive_named(int idx) {
  switch (idx) {
    case 0: bar_arrive_id<BASE>(); break;
    case 1: bar_arrive_id<BASE + 1>(); break;
    case 2: if (kTBuf > 2) bar_arrive_id<BASE + (kTBuf > 2 ? 2 : 0)>(); break;
    default: if (kTBuf > 3) bar_arrive_id<BASE + (kTBuf > 3 ? 3 : 0)>(); break;
  }
}

// Stage layout: the weights of one 32-row sub-tile (two 16-row halves, w1 then w3, for SwiGLU) as 8 K-blocks of
// [half rows][128 B] per half, 128B-swizzled; then the weight scales [32 rows][gpc floats].
// Issued by the chain warp. With k-block maps lane 0 (and lane 1 for w3) moves a whole half in one instruction;
// otherwise lanes b < 8 (and 16 + b) move one [rows x 128 B] box each. Lanes 30/31 load the scale box(es). Every box
// is copied whole (rows past the sub-tile are the next rows of the segment, or the tensor map's zero fill past the
// matrix), so the transaction count is fixed per stage.
__device__ __forceinline__ void issue_stage(const GemvMaps &m, int gpc, int kblock, const Sub &t, int chunk, bool swiglu,
                                            int lane, uint8_t *buf, uint64_t *bar) {
  if (lane == 0)
    mbar_arrive_expect_tx(bar, (unsigned)(kWeightStage + kTileRows * gpc * 4));
  __syncwarp();
  const int half = swiglu ? kTileRows / 2 : kTileRows;
  const int kb_stride = half * kBoxCols;
  const CUtensorMap *w = swiglu ? &m.wmap[0] : &m.wmap[0] + t.seg;
  const CUtensorMap *sm = swiglu ? &m.smap[0] : &m.smap[0] + t.seg;
  if (kblock) {
    if (lane == 0)
      tma_load_3d(buf, w, 0, t.row0, chunk * kBoxes, bar);
    if (swiglu && lane == 1)
      tma_load_3d(buf + half * kChunk, &m.w3map, 0, t.row0, chunk * kBoxes, bar);
  } else {
    const int x0 = chunk * kChunk;
    if (lane < kBoxes)
      tma_load_2d(buf + lane * kb_stride, w, x0 + lane * kBoxCols, t.row0, bar);
    else if (swiglu && lane >= 16 && lane < 16 + kBoxes)
      tma_load_2d(buf + half * kChunk + (lane - 16) * kb_stride, &m.w3map, x0 + (lane - 16) * kBoxCols, t.row0, bar);
  }
  if (lane == 31)
    tma_load_2d(buf + kWeightStage, sm, chunk * gpc, t.row0, bar);
  if (swiglu && lane == 30)
    tma_load_2d(buf + kWeightStage + half * gpc * 4, &m.s3map, chunk * gpc, t.row0, bar);
}

// Byte offset inside a stage of the 16-byte piece `k16` (0 .. 63 along K) of physical row r (0 .. 31): its half,
// its K-block k16 / 8, its row within the half, then the 128B swizzle (piece index XOR row within the 8-row atom).
template <int HALF>
__device__ __forceinline__ int piece_offset(int r, int k16) {
  return (r >= HALF ? HALF * kChunk : 0) + (k16 >> 3) * (HALF * kBoxCols) + (r & (HALF - 1)) * kBoxCols +
         (((k16 & 7) ^ (r & 7)) << 4);
}

// Exact int32 dot of group g of physical row r with the activations (4 independent dp4a chains for gs 64).
template <int GS, int HALF>
__device__ __forceinline__ int group_dot(const uint8_t *buf, const int8_t *xrow, int r, int g, int gs) {
  if (GS == 64) {
    int4 w[4], x[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      w[q] = lds128(buf + piece_offset<HALF>(r, g * 4 + q));
      x[q] = lds128(xrow + g * 64 + q * 16);
    }
    int d0 = dot16(w[0], x[0], 0), d1 = dot16(w[1], x[1], 0), d2 = dot16(w[2], x[2], 0), d3 = dot16(w[3], x[3], 0);
    return (d0 + d1) + (d2 + d3);
  }
  int dot = 0;
  for (int q = 0; q < gs / 16; q++)
    dot = dot16(lds128(buf + piece_offset<HALF>(r, g * (gs / 16) + q)), lds128(xrow + g * gs + q * 16), dot);
  return dot;
}

// Copies n floats from global to shared memory with all the CTA's threads, each keeping kStageBatch 16-byte loads in
// flight before its first store (a load-then-store loop would wait one memory round trip per element). L2-coherent
// loads (ld.global.cg) when `coherent`: the data may have been written by other CTAs of this very launch.
constexpr int kStageBatch = 8;

__device__ __forceinline__ void stage_floats(float *dst, const float *src, int n, bool coherent) {
  const int tid = threadIdx.x;
  if (((uintptr_t)src & 15) == 0 && (n & 3) == 0) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 *d4 = reinterpret_cast<float4 *>(dst);
    const int n4 = n / 4;
    for (int base = tid; base < n4; base += kThreads * kStageBatch) {
      float4 r[kStageBatch];
#pragma unroll
      for (int b = 0; b < kStageBatch; b++) {
        const int i = base + b * kThreads;
        if (i < n4)
          r[b] = coherent ? __ldcg(s4 + i) : __ldg(s4 + i);
      }
#pragma unroll
      for (int b = 0; b < kStageBatch; b++) {
        const int i = base + b * kThreads;
        if (i < n4)
          d4[i] = r[b];
      }
    }
  } else {
    for (int base = tid; base < n; base += kThreads * kStageBatch) {
      float r[kStageBatch];
#pragma unroll
      for (int b = 0; b < kStageBatch; b++) {
        const int i = base + b * kThreads;
        if (i < n)
          r[b] = coherent ? __ldcg(src + i) : __ldg(src + i);
      }
#pragma unroll
      for (int b = 0; b < kStageBatch; b++) {
        const int i = base + b * kThreads;
        if (i < n)
          dst[i] = r[b];
      }
    }
  }
}

// Quantizes the n staged values XF (RMS-normalized first with NW and inv when norm) in gs-groups by k_quantize's rule
// into q / s (shared or global memory), with all the CTA's threads.
__device__ __forceinline__ void quantize_staged(const float *XF, const float *NW, float inv, bool norm, int8_t *q,
                                                float *s, int n, int gs) {
  const int tid = threadIdx.x, lane = tid & 31;
  // Four lanes per group, each taking every fourth value (gs / 4 of them), the walk rotated by the group's place in
  // the warp so the 32 lanes read 32 different banks; the group max comes from two shuffles. The max is
  // order-independent and each value is quantized on its own, so the mapping does not change a bit of the result.
  const int per = gs / 4, sub = lane & 3, g8 = (lane >> 2) & 7;
  const int groups = n / gs, slots = (groups + 7) / 8 * 32;  // 8 groups per warp-sized slot
  for (int t = tid; t < slots; t += kThreads) {
    const int grp = (t >> 5) * 8 + g8;
    const bool live = grp < groups;
    const float *xg = XF + grp * gs, *wg = NW + grp * gs;
    float mx = 0.0f;
    int bad = 0;
    if (live)
      for (int i = 0; i < per; i++) {
        const int j = (4 * (i + g8) + sub) & (gs - 1);
        const float v = norm ? rms_apply(xg[j], wg[j], inv) : xg[j];
        bad |= !isfinite(v);
        mx = fmaxf(mx, fabsf(v));
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    if (!live)
      continue;
    if (bad)
      kc_raise(KC_ERR_NONFINITE);
    const float scale = __fdiv_rn(mx, 127.0f);
    if (sub == 0)
      s[grp] = scale;
    for (int i = 0; i < per; i++) {
      const int j = (4 * (i + g8) + sub) & (gs - 1);
      q[grp * gs + j] = (int8_t)quantize_value(norm ? rms_apply(xg[j], wg[j], inv) : xg[j], scale);
    }
  }
}

// The activation of the fused modes, built by all threads while the first weight stages stream in: x (and the norm
// weights) staged into shared memory, RMSNorm (the k_rmsnorm_q8_rows arithmetic: rms_lane_sum, rms_inverse,
// rms_apply) when asked, then each gs-group quantized by k_quantize's rule into XQ / XS. Bitwise the separate kernels'
// result. scratch: 65 floats (the chain buffers, unused until the main loop).
__device__ __forceinline__ void prepare_activation(const GemvArgs &a, int8_t *XQ, float *XS, float *XF, float *scratch,
                                                   int gs) {
  const int tid = threadIdx.x, n = a.n;
  const bool norm = a.act == kActNormQuantize;
  float *NW = XF + n;
  stage_floats(XF, a.xf, n, false);
  if (norm)
    stage_floats(NW, a.normw, n, false);
  __syncthreads();
  if (norm) {
    if (tid < 64)
      scratch[tid] = rms_lane_sum(XF, n, tid);
    __syncthreads();
    if (tid == 0)
      scratch[64] = rms_inverse(scratch, n, a.eps);
    __syncthreads();
  }
  quantize_staged(XF, NW, norm ? scratch[64] : 1.0f, norm, XQ, XS, n, gs);
}

// Completion counter of the tail GEMVs: every CTA adds one when its outputs are written; the one that makes it
// gridDim.x runs the tail and puts it back to zero for the next launch.
__device__ unsigned kc_gemv_tail_counter;

// The tail job (see KcGemvTail), by all the threads of the last CTA, with `scratch` (the CTA's stage buffers, free
// once its main loop is done) for staging.
__device__ void run_tail(const KcGemvTail &t, float *scratch, int gs) {
  const int tid = threadIdx.x;
  if (t.kind == KC_TAIL_ROPE_KV_STORE) {
    // k_rope_kv_store_rows for one row at *pos (rope_store_kernel's arithmetic).
    const int pos = *t.pos, half = t.hd / 2;
    if (pos < 0 || pos >= t.seq) {
      if (tid == 0)
        kc_raise(KC_ERR_BAD_ARGS);
      return;
    }
    const float *tb = t.table + (long long)pos * 2 * t.hd;
    const int nq = t.nh * t.hd, nkv = t.nkv * t.hd;
    float *Qs = scratch, *Ks = Qs + nq, *Vs = Ks + nkv;
    stage_floats(Qs, t.qv, nq, true);
    stage_floats(Ks, t.kv, nkv, true);
    stage_floats(Vs, t.vv, nkv, true);
    __syncthreads();
    const int rot = (t.nh + t.nkv) * half;
    for (int p = tid; p < rot + nkv; p += kThreads) {
      if (p < rot) {
        const bool is_k = p >= t.nh * half;
        const int pp = is_k ? p - t.nh * half : p, h = pp / half, j = 2 * (pp - h * half);
        const float *src = (is_k ? Ks : Qs) + h * t.hd + j;
        const float c = tb[j], sn = tb[t.hd + j + 1];
        const float a = src[0], b = src[1];
        const float o0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
        const float o1 = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
        float *dst = is_k ? t.kcache + ((long long)h * t.seq + pos) * t.hd + j : t.qv + h * t.hd + j;
        dst[0] = o0, dst[1] = o1;
      } else {
        const int i = p - rot, h = i / t.hd, d = i - h * t.hd;
        t.vcache[((long long)h * t.seq + pos) * t.hd + d] = Vs[i];
      }
    }
    return;
  }
  // (RMSNorm +) quantize t.x: staged through shared memory as the fused-input prologue does (same arithmetic).
  const bool norm = t.kind == KC_TAIL_NORM_QUANTIZE;
  float *XF = scratch, *NW = scratch + t.n, *lanes = NW + (norm ? t.n : 0);
  stage_floats(XF, t.x, t.n, true);
  if (norm)
    stage_floats(NW, t.w, t.n, false);
  __syncthreads();
  if (norm) {
    if (tid < 64)
      lanes[tid] = rms_lane_sum(XF, t.n, tid);
    __syncthreads();
    if (tid == 0)
      lanes[64] = rms_inverse(lanes, t.n, t.eps);
    __syncthreads();
  }
  quantize_staged(XF, NW, norm ? lanes[64] : 1.0f, norm, t.q, t.s, t.n, gs);
}

// Per-group completion counters of KC_TAIL_QUANTIZE_OUTPUT: each CTA adds the rows it wrote to every gs-group they
// touch; the CTA that brings a group to gs quantizes it and puts the counter back to zero for the next launch.
constexpr int kMaxOutputGroups = 1 << 16;
__device__ unsigned kc_gemv_group_counter[kMaxOutputGroups];

// KC_TAIL_QUANTIZE_OUTPUT for output rows [r0, r1) of `out`, which this CTA has written: count them in, then quantize
// (k_quantize's rule, one warp per group) each group this CTA completed. `flags`: shared scratch, one int per group
// the range touches.
__device__ void quantize_output_groups(const KcGemvTail &t, const float *out, int r0, int r1, int gs, int *flags) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g0 = r0 / gs, ng = (r1 - 1) / gs - g0 + 1;
  __threadfence();  // this CTA's outputs, visible before the counts say so
  __syncthreads();
  for (int i = tid; i < ng; i += kThreads) {
    const int g = g0 + i, lo = max(r0, g * gs), hi = min(r1, (g + 1) * gs);
    flags[i] = atomicAdd(&kc_gemv_group_counter[g], (unsigned)(hi - lo)) + (unsigned)(hi - lo) == (unsigned)gs;
  }
  __syncthreads();
  for (int i = warp; i < ng; i += kThreads / 32) {
    if (!flags[i])
      continue;
    const int g = g0 + i;
    __threadfence();  // the other CTAs' rows of the group, counted in before the count completed
    float mx = 0.0f;
    int bad = 0;
    for (int j = lane; j < gs; j += 32) {
      const float v = __ldcg(out + (long long)g * gs + j);
      bad |= !isfinite(v);
      mx = fmaxf(mx, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (__any_sync(0xffffffffu, bad)) {
      if (lane == 0)
        kc_raise(KC_ERR_NONFINITE);
    } else {
      const float scale = __fdiv_rn(mx, 127.0f);
      if (lane == 0)
        t.s[g] = scale;
      for (int j = lane; j < gs; j += 32)
        t.q[(long long)g * gs + j] = (int8_t)quantize_value(__ldcg(out + (long long)g * gs + j), scale);
    }
    if (lane == 0)
      kc_gemv_group_counter[g] = 0;
  }
}

// Counts this CTA's outputs in; the CTA that completes the count runs the tail. `flag`: one int of shared memory.
__device__ __forceinline__ void finish_tail(const GemvArgs &a, float *scratch, int *flag) {
  __threadfence();  // this CTA's output writes, visible before the count says so
  __syncthreads();
  if (threadIdx.x == 0)
    *flag = atomicAdd(&kc_gemv_tail_counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!*flag)
    return;
  __threadfence();
  run_tail(a.tail, scratch, a.gs);
  if (threadIdx.x == 0)
    kc_gemv_tail_counter = 0;
}

// ---- KC_REDUCE_ADD: the tensor-parallel sum inside the GEMV ------------------------------------------------------
// Every rank computes the same rows of its own column slice of the weights; the chain warp sends each finished row to
// every rank as one 8-byte {float bits, call number} store (slot [parity][rank][row] of that rank's region, over
// NVLink for the peers). Once its own rows are sent, each CTA waits, bounded, until its rows from every rank have
// arrived in this GPU's region and adds them to the output in rank order: out[r] + (((p_0 + p_1) + p_2) + ...), the
// order and rounding of kd_peer_allreduce_add after a PARTIAL GEMV, so the replicated residual stays identical on all
// ranks. The call number seq (this CTA's counter + 1) selects the parity: a rank can only start call seq + 2 after
// every rank has sent its rows of call seq + 1, which each does only after its call seq kernel finished, so a slot is
// never overwritten while it is still being read. The CTAs of one GPU never wait on each other.
__device__ __forceinline__ void push_row(const KcPeerGemv &p, long long par, unsigned seq, int row, float v) {
  const unsigned long long w = ((unsigned long long)seq << 32) | __float_as_uint(v);
  const long long off = (par * p.world + p.rank) * p.stride + row;
#pragma unroll
  for (int q = 0; q < kPeerMaxRanks; q++)  // static indices: the pointers stay in parameter space
    if (q < p.world)
      peer_st_slot(p.slots[q] + off, w);
}

__device__ __forceinline__ void reduce_rows(const KcPeerGemv &p, float *out, int r0, int r1, long long par,
                                            unsigned seq) {
  const unsigned long long *mine = p.slots[0];
#pragma unroll
  for (int q = 1; q < kPeerMaxRanks; q++)
    mine = q == p.rank ? p.slots[q] : mine;
  mine += par * p.world * p.stride;
  const uint64_t start = kc_globaltimer();
  for (int r = r0 + (int)threadIdx.x; r < r1; r += (int)blockDim.x) {
    float sum = 0.0f;
    bool ok = true;
    for (int q = 0; q < p.world && ok; q++) {
      unsigned long long v = peer_ld_slot(mine + q * p.stride + r);
      for (unsigned k = 1; (unsigned)(v >> 32) != seq; k++) {
        if ((k & 63u) == 0 && kc_globaltimer() - start > KC_WAIT_NS) {
          kc_raise(KC_ERR_TIMEOUT);
          ok = false;
          break;
        }
        v = peer_ld_slot(mine + q * p.stride + r);
      }
      const float f = __uint_as_float((unsigned)v);
      sum = q == 0 ? f : __fadd_rn(sum, f);
    }
    if (ok)
      out[r] = __fadd_rn(out[r], sum);
  }
}

// RED: the KC_REDUCE_ADD instantiation; the others carry none of its code.
template <int GS, bool RED>
__global__ void __launch_bounds__(kThreads, 1) gemv_q8_kernel(const __grid_constant__ GemvMaps m, const GemvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  // The 128-byte swizzle is a function of the address bits, so the stages start on a 1024-byte boundary.
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  pdl_launch_dependents();
  const bool swiglu = a.kind == KC_SWIGLU;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, c = blockIdx.x;
  const int u0 = a.units * c / G, u1 = a.units * (c + 1) / G;  // units * grid < 2^31 (checked on the host)
  if (u1 <= u0) {
    if (a.tail.kind && a.tail.kind != KC_TAIL_QUANTIZE_OUTPUT)
      finish_tail(a, reinterpret_cast<float *>(smem), reinterpret_cast<int *>(smem));
    if (RED) {  // no rows, but the call still counts
      pdl_wait();
      if (tid == 0)
        a.peer.epoch[c] += 1u;
    }
    return;
  }
  const Plan plan = make_plan(a, u0, u1, swiglu ? 4 : 5);
  const int nchunks = a.nchunks, depth = a.depth, stage_bytes = a.stage_bytes, n = a.n;
  const int S = (plan.nsub[0] + plan.nsub[1] + plan.nsub[2]) * nchunks;
  const int gs = GS ? GS : a.gs;
  const int gpc = kChunk / gs;
  float *const out0 = a.seg[0].out, *const out1 = a.seg[1].out, *const out2 = a.seg[2].out;

  // Shared memory: the stages (1024-byte aligned for the swizzle), then barriers, flags, chain buffers, activations.
  uint8_t *stages = smem;
  uint8_t *tail = smem + depth * stage_bytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(tail);
  volatile int *abort_flag = reinterpret_cast<int *>(tail + 8 * 8);
  volatile int *issued = reinterpret_cast<int *>(tail + 8 * 8 + 4);
  float *T = reinterpret_cast<float *>(tail + 128);
  float *XS = T + kTBuf * gpc * kTileRows;
  int8_t *XQ = reinterpret_cast<int8_t *>(XS + ((n / gs + 3) & ~3));

  if (tid == 0) {
    for (int i = 0; i < depth; i++)
      mbar_init(&bars[i], 1);
    *abort_flag = 0;
    *issued = min(depth, S);
    fence_mbar_init();
  }
  __syncthreads();
  // Weights do not depend on the previous kernel: the first stage streams in before waiting for it. The others are
  // issued once the activation loads are on their way, so those few kilobytes do not queue behind the whole
  // prefetch on the way into this SM.
  if (warp == kDotWarps && S > 0)
    issue_stage(m, gpc, a.kblock, subtile(plan, 0), 0, swiglu, lane, stages, &bars[0]);
  pdl_wait();
  // The counter was written by the previous reducing call, complete once pdl_wait returns.
  const unsigned seq = RED ? a.peer.epoch[c] + 1u : 0u;
  const long long par = seq & 1u;
  if (a.act == kActQ8) {
    for (int i = tid; i < n / 16; i += kThreads)
      reinterpret_cast<int4 *>(XQ)[i] = __ldg(reinterpret_cast<const int4 *>(a.xq) + i);
    for (int i = tid; i < n / gs; i += kThreads)
      XS[i] = __ldg(a.xs + i);
  } else {
    prepare_activation(a, XQ, XS, reinterpret_cast<float *>(XQ + ((n + 15) & ~15)), T, gs);
  }
  if (warp == kDotWarps)
    for (int i = 1; i < depth && i < S; i++)
      issue_stage(m, gpc, a.kblock, subtile(plan, i / nchunks), i % nchunks, swiglu, lane, stages + i * stage_bytes,
                  &bars[i]);
  __syncthreads();

  if (warp < kDotWarps) {
    // ---- dot warps: exact int32 group dots of 32 rows, scaled by the activation scale, into T[stage & 1] ----
    int slot = 0, chunk = 0, sub = 0;
    unsigned phase = 0;
    for (int i = 0; i < S; i++) {
      const Sub t = subtile(plan, sub);
      if (!*abort_flag && !mbar_wait_bounded(&bars[slot], phase))
        *abort_flag = 1;
      if (i >= kTBuf)
        bar_sync_named<kBarTEmpty>(i % kTBuf);
      const uint8_t *buf = stages + slot * stage_bytes;
      float *Tb = T + (i % kTBuf) * gpc * kTileRows;
      const int groups = min(gpc, (n - chunk * kChunk) / gs);
      if (lane_active(swiglu, lane, t.cnt)) {
        const int8_t *xrow = XQ + chunk * kChunk;
        const float *xsc = XS + chunk * gpc;
        if (GS == 64 && groups == kFastGroups) {
          // All of this warp's groups at once: 4 independent dp4a chains per group in flight.
          int d[kWarpGroups];
#pragma unroll
          for (int j = 0; j < kWarpGroups; j++)
            d[j] = swiglu ? group_dot<GS, 16>(buf, xrow, lane, warp + j * kDotWarps, gs)
                          : group_dot<GS, 32>(buf, xrow, lane, warp + j * kDotWarps, gs);
#pragma unroll
          for (int j = 0; j < kWarpGroups; j++)
            Tb[(warp + j * kDotWarps) * kTileRows + lane] =
                __fmul_rn(__int2float_rn(d[j]), xsc[warp + j * kDotWarps]);
        } else {
          for (int g = warp; g < groups; g += kDotWarps) {
            const int d = swiglu ? group_dot<GS, 16>(buf, xrow, lane, g, gs) : group_dot<GS, 32>(buf, xrow, lane, g, gs);
            Tb[g * kTileRows + lane] = __fmul_rn(__int2float_rn(d), xsc[g]);
          }
        }
      }
      bar_arrive_named<kBarTFull>(i % kTBuf);
      if (++slot == depth)
        slot = 0, phase ^= 1u;
      if (++chunk == nchunks)
        chunk = 0, sub++;
    }
  } else {
    // ---- chain warp: the ordered fp32 accumulation (one lane per row), the epilogue, and the TMA producer ----
    float acc = 0.0f;
    int slot = 0, chunk = 0, sub = 0;
    int nchunk = depth % nchunks, nsub = depth / nchunks;  // chunk and sub-tile of stage i + depth
    for (int i = 0; i < S; i++) {
      const Sub t = subtile(plan, sub);
      bar_sync_named<kBarTFull>(i % kTBuf);
      const float *Tb = T + (i % kTBuf) * gpc * kTileRows;
      const float *wsr = reinterpret_cast<const float *>(stages + slot * stage_bytes + kWeightStage) + lane * gpc;
      const int groups = min(gpc, (n - chunk * kChunk) / gs);
      if (GS == 64 && groups == kFastGroups && lane_active(swiglu, lane, t.cnt)) {
        // 16 groups at a time: their scaled dots and weight scales loaded first, then the 16 dependent FMAs.
#pragma unroll
        for (int h = 0; h < kFastGroups; h += 16) {
          float tv[16], wv[16];
#pragma unroll
          for (int g = 0; g < 16; g += 4) {
            float4 w4 = *reinterpret_cast<const float4 *>(wsr + h + g);
            wv[g] = w4.x, wv[g + 1] = w4.y, wv[g + 2] = w4.z, wv[g + 3] = w4.w;
          }
#pragma unroll
          for (int g = 0; g < 16; g++)
            tv[g] = Tb[(h + g) * kTileRows + lane];
#pragma unroll
          for (int g = 0; g < 16; g++)
            acc = __fmaf_rn(tv[g], wv[g], acc);
        }
      } else if (lane_active(swiglu, lane, t.cnt)) {
        for (int g = 0; g < groups; g += 4) {
          float4 w4 = *reinterpret_cast<const float4 *>(wsr + g);
          acc = __fmaf_rn(Tb[g * kTileRows + lane], w4.x, acc);
          if (g + 1 < groups)
            acc = __fmaf_rn(Tb[(g + 1) * kTileRows + lane], w4.y, acc);
          if (g + 2 < groups)
            acc = __fmaf_rn(Tb[(g + 2) * kTileRows + lane], w4.z, acc);
          if (g + 3 < groups)
            acc = __fmaf_rn(Tb[(g + 3) * kTileRows + lane], w4.w, acc);
        }
      }
      if (chunk == nchunks - 1) {
        float gate = __shfl_down_sync(0xffffffffu, acc, 16);
        float *out = (t.seg == 0 ? out0 : t.seg == 1 ? out1 : out2) + t.row0;
        if (swiglu) {
          if (lane < t.cnt)
            out[lane] = silu_gate_dev(acc, gate);
        } else if (lane < t.cnt) {
          if (a.kind == KC_ADD)
            out[lane] = __fadd_rn(out[lane], acc);
          else if (RED)
            push_row(a.peer, par, seq, t.row0 + lane, acc);
          else
            out[lane] = acc;
        }
        acc = 0.0f;
      }
      // Stage i is fully consumed (dot warps passed T_FULL after their last read of its weights, and the chain has
      // read its scales): refill the slot with stage i + depth.
      if (i + depth < S && !*abort_flag) {
        issue_stage(m, gpc, a.kblock, subtile(plan, nsub), nchunk, swiglu, lane, stages + slot * stage_bytes,
                    &bars[slot]);
        if (lane == 0)
          *issued = i + depth + 1;
      }
      if (++nchunk == nchunks)
        nchunk = 0, nsub++;
      if (i + kTBuf < S)
        bar_arrive_named<kBarTEmpty>(i % kTBuf);
      if (++slot == depth)
        slot = 0;
      if (++chunk == nchunks)
        chunk = 0, sub++;
    }
  }
  // After an abort, let every copy still in flight land (bounded waits) before the shared memory goes away: for each
  // slot, the latest stage issued into it.
  __syncthreads();
  if (*abort_flag && tid == 0)
    for (int j = max(0, *issued - depth); j < *issued; j++)
      mbar_wait_bounded(&bars[j % depth], (unsigned)(j / depth) & 1u);
  if (RED) {
    reduce_rows(a.peer, out0, u0, u1, par, seq);
    __syncthreads();
    if (tid == 0)
      a.peer.epoch[c] = seq;
  }
  if (a.tail.kind == KC_TAIL_QUANTIZE_OUTPUT) {
    __syncthreads();
    quantize_output_groups(a.tail, out0, u0, u1, gs, reinterpret_cast<int *>(stages));
  } else if (a.tail.kind) {
    __syncthreads();
    finish_tail(a, reinterpret_cast<float *>(stages), const_cast<int *>(abort_flag) + 2);
  }
}

// The general rung, for shapes the TMA kernel cannot describe (group sizes below 16 or not a power of two, scale rows
// that are not 16-byte multiples, unaligned pointers): one warp per output row, the group dot reduced exactly across
// the warp, lane 0 applying the same ordered rescale. Slow but bitwise identical to the fast kernel.
__global__ void __launch_bounds__(256) gemv_q8_generic_kernel(GemvSegDev s0, GemvSegDev s1, GemvSegDev s2,
                                                               const int8_t *wq0, const int8_t *wq1, const int8_t *wq2,
                                                               const float *ws0, const float *ws1, const float *ws2,
                                                               const int8_t *w3q, const float *w3s, int nseg,
                                                               const int8_t *xq, const float *xs, int n, long long ld,
                                                               int gs, int kind, int units) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int unit = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (unit >= units)
    return;
  int s = (nseg > 1 && unit >= s1.unit0) ? 1 : 0;
  if (nseg > 2 && unit >= s2.unit0)
    s = 2;
  const GemvSegDev seg = s == 0 ? s0 : s == 1 ? s1 : s2;
  const int row = unit - seg.unit0;
  const int8_t *wq = (s == 0 ? wq0 : s == 1 ? wq1 : wq2) + row * ld;
  const float *ws = (s == 0 ? ws0 : s == 1 ? ws1 : ws2) + row * (ld / gs);
  float acc[2] = {0.0f, 0.0f};
  for (int pass = 0; pass < (kind == KC_SWIGLU ? 2 : 1); pass++) {
    const int8_t *w = pass ? w3q + row * ld : wq;
    const float *sc = pass ? w3s + row * (ld / gs) : ws;
    for (int g = 0; g < n / gs; g++) {
      int dot = 0;
      for (int k = lane; k < gs; k += 32)
        dot += (int)xq[g * gs + k] * (int)w[g * gs + k];
#pragma unroll
      for (int o = 16; o; o >>= 1)
        dot += __shfl_xor_sync(0xffffffffu, dot, o);
      acc[pass] = __fmaf_rn(__fmul_rn(__int2float_rn(dot), xs[g]), sc[g], acc[pass]);
    }
  }
  if (lane == 0) {
    float *out = seg.out + row;
    if (kind == KC_SWIGLU)
      *out = silu_gate_dev(acc[0], acc[1]);
    else if (kind == KC_ADD)
      *out = __fadd_rn(*out, acc[0]);
    else
      *out = acc[0];
  }
}

// act_floats: fp32 staging of the fused activation modes (n, or 2n with the norm weights).
size_t smem_bytes(int n, int gs, int stage_bytes, int depth, int act_floats) {
  return (size_t)depth * stage_bytes + 128 + (size_t)kTBuf * (kChunk / gs) * kTileRows * 4 + (size_t)((n / gs + 3) & ~3) * 4 +
         (size_t)((n + 15) & ~15) + (size_t)act_floats * 4 + 1024;
}

bool encode_weight(CUtensorMap *wmap, CUtensorMap *smap, const int8_t *wq, const float *ws, int rows, int n,
                   long long ld, int gs, int box_rows, bool kblock) {
  const int gpc = kChunk / gs;
  bool ok = kblock ? kc_tmap_kblocks(wmap, wq, (uint64_t)n, (uint64_t)rows, (uint64_t)ld, kBoxes, box_rows)
                   : kc_tmap_2d(wmap, wq, 1, (uint64_t)n, (uint64_t)rows, (uint64_t)ld, kBoxCols, box_rows, true);
  return ok &&
         kc_tmap_2d(smap, ws, 4, (uint64_t)(n / gs), (uint64_t)rows, (uint64_t)(ld / gs) * 4, gpc, box_rows, false);
}

}  // namespace

// W8A32 (K8Input.q NULL: fp32 activations x against the int8 weights), bitwise the reference on both of its paths.
// AVX (gs % 16 == 0): its AVX-512 kernel dots_q8f_body (src/gemv.c:141-180). Each of the 16 vector lanes is a lane of
// a half-warp, one output row per half-warp: lane l sums columns c + l into ga and c + 16 + l into gb over each
// 32-column step of a group (a last 16 columns, when gs % 32 == 16, into ga), then acc = fma(ga + gb, ws[g], acc); the
// row is the 16 accumulators reduced in _mm512_reduce_add_ps's tree (pairs 8, 4, 2, 1 lanes apart).
// Otherwise: its portable loop (src/gemv.c:427-436), one thread per row: per group the products added in column order,
// then val += group * ws, no fused multiply-add.
// For SwiGLU each row is computed for w1 and for w3 and combined with silu_gate. The activations are read through the
// read-only cache: every row of the CTA reads the same ones.
template <bool AVX>
__global__ void __launch_bounds__(256) gemv_q8f_kernel(GemvSegDev s0, GemvSegDev s1, GemvSegDev s2,
                                                        const int8_t *wq0, const int8_t *wq1, const int8_t *wq2,
                                                        const float *ws0, const float *ws1, const float *ws2,
                                                        const int8_t *w3q, const float *w3s, int nseg, const float *x,
                                                        int n, long long ld, int gs, int kind, int units) {
  pdl_wait();
  const int per_cta = AVX ? (int)blockDim.x / 16 : (int)blockDim.x;
  const int l = AVX ? (int)(threadIdx.x & 15) : 0;
  const int unit = blockIdx.x * per_cta + (AVX ? (int)(threadIdx.x >> 4) : (int)threadIdx.x);
  if (!AVX && unit >= units)
    return;
  const int u = unit < units ? unit : units - 1;  // AVX: a half-warp past the end computes a real row, stores nothing
  int s = (nseg > 1 && u >= s1.unit0) ? 1 : 0;
  if (nseg > 2 && u >= s2.unit0)
    s = 2;
  const GemvSegDev seg = s == 0 ? s0 : s == 1 ? s1 : s2;
  const long long row = u - seg.unit0, sld = ld / gs;
  const int groups = n / gs;
  float res[2] = {0.0f, 0.0f};
  for (int pass = 0; pass < (kind == KC_SWIGLU ? 2 : 1); pass++) {
    const int8_t *w = (pass ? w3q : s == 0 ? wq0 : s == 1 ? wq1 : wq2) + row * ld;
    const float *sc = (pass ? w3s : s == 0 ? ws0 : s == 1 ? ws1 : ws2) + row * sld;
    float acc = 0.0f;
    if (AVX) {
      for (int g = 0; g < groups; g++) {
        const long long b = (long long)g * gs;
        float ga = 0.0f, gb = 0.0f;
        int c = 0;
        for (; c + 32 <= gs; c += 32) {
          ga = __fmaf_rn((float)w[b + c + l], __ldg(x + b + c + l), ga);
          gb = __fmaf_rn((float)w[b + c + 16 + l], __ldg(x + b + c + 16 + l), gb);
        }
        for (; c < gs; c += 16)
          ga = __fmaf_rn((float)w[b + c + l], __ldg(x + b + c + l), ga);
        acc = __fmaf_rn(__fadd_rn(ga, gb), __ldg(sc + g), acc);
      }
#pragma unroll
      for (int o = 8; o; o >>= 1)
        acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, o, 16));
    } else {
      for (int g = 0; g < groups; g++) {
        const long long b = (long long)g * gs;
        float group = 0.0f;
        for (int k = 0; k < gs; k++)
          group = __fadd_rn(group, __fmul_rn((float)w[b + k], __ldg(x + b + k)));
        acc = __fadd_rn(acc, __fmul_rn(group, __ldg(sc + g)));
      }
    }
    res[pass] = acc;
  }
  if (unit < units && l == 0) {
    float *out = seg.out + row;
    if (kind == KC_SWIGLU)
      *out = silu_gate_dev(res[0], res[1]);
    else if (kind == KC_ADD)
      *out = __fadd_rn(*out, res[0]);
    else
      *out = res[0];
  }
}

static int launch_generic(const KcGemvSeg *segs, int nseg, const int8_t *xq, const float *xs, int n, long long ld,
                          int gs, int kind, cudaStream_t stream) {
  GemvSegDev d[3] = {};
  const int8_t *wq[3] = {};
  const float *ws[3] = {};
  int units = 0;
  for (int s = 0; s < nseg; s++) {
    d[s].out = segs[s].out, d[s].d = segs[s].d, d[s].unit0 = units;
    wq[s] = segs[s].wq, ws[s] = segs[s].ws;
    units += segs[s].d;
  }
  if (units == 0 || n == 0)
    return 0;
  gemv_q8_generic_kernel<<<(units + 7) / 8, 256, 0, stream>>>(d[0], d[1], d[2], wq[0], wq[1], wq[2], ws[0], ws[1],
                                                              ws[2], segs[0].w3q, segs[0].w3s, nseg, xq, xs, n, ld, gs,
                                                              kind, units);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

static int launch_tma(const KcGemvSeg *segs, int nseg, const int8_t *xq, const float *xs, const KcGemvAct *act, int n,
                      long long ld, int gs, int kind, cudaStream_t stream, int grid_limit,
                      const KcGemvTail *tail = nullptr, const KcPeerGemv *peer = nullptr);

// The W8A32 GEMV (see gemv_q8f_kernel): 16 rows per 256-thread CTA on the AVX order, 256 on the portable one.
int kc_launch_gemv_w8a32(const KcGemvSeg *segs, int nseg, const float *x, int n, long long ld, int gs, int kind,
                         cudaStream_t stream) {
  GemvSegDev d[3] = {};
  const int8_t *wq[3] = {};
  const float *ws[3] = {};
  int units = 0;
  for (int s = 0; s < nseg; s++) {
    d[s].out = segs[s].out, d[s].d = segs[s].d, d[s].unit0 = units;
    wq[s] = segs[s].wq, ws[s] = segs[s].ws;
    units += segs[s].d;
  }
  if (units == 0 || n == 0)
    return 0;
  if (gs % 16 == 0)
    gemv_q8f_kernel<true><<<(units + 15) / 16, 256, 0, stream>>>(d[0], d[1], d[2], wq[0], wq[1], wq[2], ws[0], ws[1],
                                                                 ws[2], segs[0].w3q, segs[0].w3s, nseg, x, n, ld, gs,
                                                                 kind, units);
  else
    gemv_q8f_kernel<false><<<(units + 255) / 256, 256, 0, stream>>>(d[0], d[1], d[2], wq[0], wq[1], wq[2], ws[0],
                                                                    ws[1], ws[2], segs[0].w3q, segs[0].w3s, nseg, x, n,
                                                                    ld, gs, kind, units);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Host launcher (argument validation is the C-ABI layer's job): the TMA kernel where the shape allows it, else the
// general rung.
int kc_launch_gemv(const KcGemvSeg *segs, int nseg, const int8_t *xq, const float *xs, int n, long long ld, int gs,
                   int kind, cudaStream_t stream, int grid_limit) {
  int rc = launch_tma(segs, nseg, xq, xs, nullptr, n, ld, gs, kind, stream, grid_limit);
  if (rc == -1)
    rc = launch_generic(segs, nseg, xq, xs, n, ld, gs, kind, stream);
  return rc;
}

int kc_launch_gemv_tail(const KcGemvSeg *segs, int nseg, const int8_t *xq, const float *xs, int n, long long ld,
                        int gs, int kind, const KcGemvTail &tail, cudaStream_t stream) {
  return launch_tma(segs, nseg, xq, xs, nullptr, n, ld, gs, kind, stream, 0, &tail);
}

// The fused-activation GEMV: the TMA kernel only (-1 when the shape does not fit it).
int kc_launch_gemv_f32(const KcGemvSeg *segs, int nseg, const KcGemvAct &act, int n, long long ld, int gs, int kind,
                       cudaStream_t stream, const KcGemvTail *tail) {
  return launch_tma(segs, nseg, nullptr, nullptr, &act, n, ld, gs, kind, stream, 0, tail);
}

// The reducing GEMV: the TMA kernel only (-1 when the shape does not fit it; there is no general rung to fall back
// to, as every rank must run the same kernel).
int kc_launch_gemv_reduce(const KcGemvSeg &seg, const int8_t *xq, const float *xs, int n, long long ld, int gs,
                          const KcPeerGemv &peer, cudaStream_t stream) {
  return launch_tma(&seg, 1, xq, xs, nullptr, n, ld, gs, KC_REDUCE_ADD, stream, 0, nullptr, &peer);
}

static int launch_tma(const KcGemvSeg *segs, int nseg, const int8_t *xq, const float *xs, const KcGemvAct *act, int n,
                      long long ld, int gs, int kind, cudaStream_t stream, int grid_limit, const KcGemvTail *tail,
                      const KcPeerGemv *peer) {
  thread_local GemvMaps M;
  GemvArgs A;
  memset(&M, 0, sizeof(M));
  memset(&A, 0, sizeof(A));
  if (gs < 16 || gs > kChunk || (gs & (gs - 1)) || n % gs || ld % gs || ld < n || ((ld / gs) * 4) % 16 ||
      ((uintptr_t)xq & 15) || (act && gs > 256))
    return -1;
  int act_floats = 0;
  if (act) {
    A.xf = act->x;
    A.normw = act->norm;
    A.eps = act->eps;
    A.act = act->norm ? kActNormQuantize : kActQuantize;
    act_floats = act->norm ? 2 * n : n;
  }
  if (kind == KC_REDUCE_ADD) {
    if (!peer || nseg != 1 || tail || act || segs[0].d <= 0 || segs[0].d > peer->stride || peer->world < 1 ||
        peer->world > kPeerMaxRanks || peer->rank < 0 || peer->rank >= peer->world || !peer->epoch)
      return -1;
    A.peer = *peer;
  }
  const bool swiglu = kind == KC_SWIGLU;
  const int box_rows = swiglu ? kTileRows / 2 : kTileRows;
  int units = 0;
  for (int s = 0; s < nseg; s++) {
    A.seg[s].out = segs[s].out;
    A.seg[s].d = segs[s].d;
    A.seg[s].unit0 = units;
    units += segs[s].d;
    if (segs[s].d > 0 && (((uintptr_t)segs[s].ws & 15) || (swiglu && ((uintptr_t)segs[s].w3s & 15))))
      return -1;
  }
  // Prefer the 3-D k-block maps (one TMA instruction per stage); fall back to 2-D boxes if the driver refuses them.
  bool kblock = n % kBoxCols == 0;
  for (int attempt = 0; attempt < 2; attempt++) {
    bool ok = true;
    for (int s = 0; s < nseg && ok; s++) {
      if (segs[s].d == 0)
        continue;
      ok = encode_weight(&M.wmap[s], &M.smap[s], segs[s].wq, segs[s].ws, segs[s].d, n, ld, gs, box_rows, kblock) &&
           (!swiglu ||
            encode_weight(&M.w3map, &M.s3map, segs[s].w3q, segs[s].w3s, segs[s].d, n, ld, gs, box_rows, kblock));
    }
    if (ok)
      break;
    if (!kblock)
      return -1;
    kblock = false;
  }
  if (units == 0 || n == 0)
    return 0;
  if ((long long)units * 1024 >= (1ll << 31))
    return -1;
  A.nseg = nseg;
  A.kblock = kblock ? 1 : 0;
  A.xq = xq;
  A.xs = xs;
  A.n = n;
  A.gs = gs;
  A.kind = kind;
  A.units = units;
  A.nchunks = (n + kChunk - 1) / kChunk;
  A.stage_bytes = (kWeightStage + kTileRows * (kChunk / gs) * 4 + 1023) & ~1023;
#ifndef KC_GEMV_SMEM_BUDGET
#define KC_GEMV_SMEM_BUDGET (200 * 1024)
#endif
#ifndef KC_GEMV_MAX_DEPTH
#define KC_GEMV_MAX_DEPTH 4
#endif
  // The fused modes may use the rest of the 227 KB for their fp32 staging rather than give up pipeline depth.
  size_t budget = act ? 226 * 1024 : KC_GEMV_SMEM_BUDGET;
  if (smem_bytes(n, gs, A.stage_bytes, 2, act_floats) > budget)
    budget = 226 * 1024;
  if (smem_bytes(n, gs, A.stage_bytes, 2, act_floats) > budget)
    return -1;
  int depth = 2;
  while (depth < KC_GEMV_MAX_DEPTH && smem_bytes(n, gs, A.stage_bytes, depth + 1, act_floats) <= budget)
    depth++;
  A.depth = depth;
  const size_t smem = smem_bytes(n, gs, A.stage_bytes, depth, act_floats);
  if (tail) {
    // The tail stages its vector (and the norm weights) in the stage buffers.
    const int tail_floats = tail->kind == KC_TAIL_NORM_QUANTIZE   ? 2 * tail->n + 65
                            : tail->kind == KC_TAIL_QUANTIZE      ? tail->n
                            : tail->kind == KC_TAIL_ROPE_KV_STORE ? (tail->nh + 2 * tail->nkv) * tail->hd
                                                                  : 0;
    if ((size_t)tail_floats * 4 > (size_t)depth * A.stage_bytes || (tail->kind <= KC_TAIL_NORM_QUANTIZE &&
                                                                    tail->kind && (tail->n % gs || gs > 256)))
      return -1;
    // The output quantizer: one STORE or SwiGLU segment of whole groups, within the counters.
    if (tail->kind == KC_TAIL_QUANTIZE_OUTPUT &&
        (nseg != 1 || (kind != KC_STORE && kind != KC_SWIGLU) || segs[0].d % gs || segs[0].d / gs > kMaxOutputGroups ||
         !tail->q || !tail->s))
      return -1;
    A.tail = *tail;
  }
  const int sms = kc_device_sms();
  int grid = units < sms ? units : sms;
  if (grid_limit > 0 && grid > grid_limit)
    grid = grid_limit;
  if (kind == KC_REDUCE_ADD)  // one grid size for every call: each CTA's counter counts every call
    grid = sms < kPeerGemvMaxCtas ? sms : kPeerGemvMaxCtas;
  static bool attr_set[64][4];
  int dev = 0;
  cudaGetDevice(&dev);
  const int variant = (gs == 64 ? 0 : 1) + (kind == KC_REDUCE_ADD ? 2 : 0);
  void (*const kernels[4])(const GemvMaps, const GemvArgs) = {gemv_q8_kernel<64, false>, gemv_q8_kernel<0, false>,
                                                              gemv_q8_kernel<64, true>, gemv_q8_kernel<0, true>};
  if (dev < 64 && !attr_set[dev][variant]) {
    cudaFuncSetAttribute(kernels[variant], cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr_set[dev][variant] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = kc_pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernels[variant], M, A);
  return e == cudaSuccess ? 0 : -2;
}
