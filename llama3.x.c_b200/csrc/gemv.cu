// Q8_0 W8A8 decode GEMV for sm_100a: y[r] = sum over groups g of (float)dot_g(xq, wq[r]) * xs[g] * ws[r][g] with the
// epilogues of the reference's GEMV drivers (src/gemv.c:441-528: STORE / ADD / PARTIAL over 1-3 segments, SWIGLU on
// a w1/w3 pair).
//
// Arithmetic: the reference's AVX-512 W8A8 kernel, dots_q8_body (src/gemv.c:109-139), which its k_matmul_q8 runs for
// gs % 64 == 0 on every AVX-512 host. A row is 16 vector lanes; lane L (0..15) owns bytes 4L..4L+3 of every 64-byte
// piece of the row. Per group g its int32 sum is exact (vpdpbusd with |x| and sign(x)·w is the signed dot, since no
// int8 value is -128), and it is rescaled into the lane's own fp32 accumulator:
//   acc[L] = fmaf((float)dot_L(g) * xs[g], ws[r][g], acc[L])      for g = 0, 1, ..., ascending, from acc = 0
// The row's result is the 16 accumulators reduced in _mm512_reduce_add_ps's tree (lanes 8 apart, then 4, 2, 1). The
// output is therefore bitwise the reference's decode GEMV.
//
// Work split: 8 threads per weight row, thread j holding the accumulators of lanes 2j and 2j+1 (one dp4a each per
// 64-byte piece; the int32 lane sum is turned into its exact float by adding 1.5·2^23 inside the dp4a and
// subtracting it in fp32, cheaper than a conversion instruction). So every thread carries its own two ordered chains
// through the whole row and no partial result crosses a warp: the 16-lane tree at the end of the row is three
// shuffles within 8 lanes.
//
// Data movement: the weight bytes are HBM-bound. Each CTA owns a contiguous range of output rows in whole octets (8
// rows), walks it in sub-tiles of 32 physical weight rows that never straddle a segment, and streams each sub-tile
// through shared memory in 1 KiB K-chunks with TMA tensor copies: per octet of rows one 3-D box [8 K-blocks x 8 rows x
// 128 B] (128-byte swizzled; only the octets the sub-tile covers are read, so no row is read by two CTAs), plus one
// box of the chunk's weight scales, completing on the stage's full barrier, several stages deep. A producer warp
// refills a stage once the 8 compute warps have arrived on its empty barrier; nothing else synchronises the loop.
// Bank conflicts: the 8 threads of a row read 64 contiguous bytes (4 swizzled 16-byte pieces), and the two rows of a
// half-warp are 4 apart within their 8-row swizzle atom, so they hit the other 4 pieces.
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

constexpr int kComputeWarps = 8;
constexpr int kThreads = (kComputeWarps + 1) * 32;  // 8 compute warps + 1 TMA producer warp
constexpr int kTileRows = 32;                       // physical weight rows per sub-tile (4 per compute warp)
constexpr int kOctRows = 8;                         // weight rows per TMA box: one 1024-byte swizzle atom per K-block
constexpr int kChunk = 1024;                        // K bytes per stage
constexpr int kBoxCols = 128;                       // bytes per 128B-swizzled box row
constexpr int kBoxes = kChunk / kBoxCols;           // K-blocks per chunk
constexpr int kOctBytes = kOctRows * kChunk;        // one octet of rows over a chunk
constexpr int kWeightStage = kTileRows * kChunk;
constexpr int kMaxDepth = 8;
constexpr int kCtrlBytes = 512;  // full and empty barriers, flags, 65 floats of prologue scratch
// 1.5 * 2^23: an int32 v with |v| < 2^22 added to these bits reads as the float 12582912 + v exactly.
constexpr int kMagicBits = 0x4B400000;
constexpr float kMagic = 12582912.0f;

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


// Stage layout: four octet slots of [8 K-blocks][8 rows][128 B] (128B-swizzled), octet o holding physical rows
// 8o..8o+7 of the sub-tile (for SwiGLU: octets 0-1 are w1's 16 rows, 2-3 w3's), then the weight scales [32 rows][gpc
// floats] (w1's 16 rows, then w3's). Issued by the producer warp. Only the octets the sub-tile's rows reach are copied
// (the scale box is always whole: rows past the matrix are zero-filled), so the transaction count is computed per
// stage. With k-block maps lanes 0-3 move one octet each in a single instruction; otherwise lane 8o + b moves K-block
// b of octet o as a [128 B x 8 rows] box. Every box is copied whole: rows and columns past the matrix are the tensor
// map's zero fill.
__device__ __forceinline__ void issue_stage(const GemvMaps &m, int gpc, int kblock, const Sub &t, int chunk, bool swiglu,
                                            int lane, uint8_t *buf, uint64_t *bar) {
  const int noct = (t.cnt + kOctRows - 1) / kOctRows;  // octets per half (SwiGLU) or per sub-tile
  const int srows = swiglu ? kTileRows / 2 : kTileRows;
  if (lane == 0)
    mbar_arrive_expect_tx(bar, (unsigned)((swiglu ? 2 * noct : noct) * kOctBytes + kTileRows * gpc * 4));
  __syncwarp();
  const int o = kblock ? lane : lane >> 3;  // the octet slot this lane serves
  const bool w3 = swiglu && o >= 2;
  const int orow = swiglu ? (o & 1) : o;  // octet index within its half
  if (o < 4 && orow < noct) {
    const CUtensorMap *w = w3 ? &m.w3map : swiglu ? &m.wmap[0] : &m.wmap[0] + t.seg;
    const int row = t.row0 + orow * kOctRows;
    if (kblock)
      tma_load_3d(buf + o * kOctBytes, w, 0, row, chunk * kBoxes, bar);
    else
      tma_load_2d(buf + o * kOctBytes + (lane & 7) * (kOctRows * kBoxCols), w, chunk * kChunk + (lane & 7) * kBoxCols,
                  row, bar);
  }
  if (lane == 31)
    tma_load_2d(buf + kWeightStage, swiglu ? &m.smap[0] : &m.smap[0] + t.seg, chunk * gpc, t.row0, bar);
  if (swiglu && lane == 30)
    tma_load_2d(buf + kWeightStage + srows * gpc * 4, &m.s3map, chunk * gpc, t.row0, bar);
}

__device__ __forceinline__ uint2 lds64(const void *p) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_u32(p)));
  return v;
}

// Byte offset, from the start of a row inside its octet slot, of the 8 bytes at K offset `kb8 * 8` of the chunk for
// a row at position `r7` of its octet: K-block, then the 16-byte piece XOR the row (the 128B swizzle), then the half
// of the piece.
__device__ __forceinline__ int row_offset(int r7, int kb8) {
  return (kb8 >> 4) * (kOctRows * kBoxCols) + ((((kb8 >> 1) & 7) ^ r7) << 4) + ((kb8 & 1) << 3);
}

// One gs-group of a chunk for this thread's two lanes: the exact int32 sums of lanes 2j and 2j+1 (one dp4a each per
// 64-byte piece, started from the magic bits), their exact floats, times xs, fused into the accumulators with ws.
template <int GS>
__device__ __forceinline__ void group_step(const uint8_t *rowbuf, int r7, const int8_t *xrow, int g, int gs, int j,
                                           float xs, float ws, float &a0, float &a1) {
  const int gsz = GS ? GS : gs;
  int d0 = kMagicBits, d1 = kMagicBits;
#pragma unroll
  for (int c = 0; c < gsz; c += 64) {
    const int kb8 = (g * gsz + c) / 8 + j;  // 8-byte unit of the chunk
    const uint2 w = lds64(rowbuf + row_offset(r7, kb8));
    const uint2 x = lds64(xrow + kb8 * 8);
    d0 = __dp4a((int)w.x, (int)x.x, d0);
    d1 = __dp4a((int)w.y, (int)x.y, d1);
  }
  const float f0 = __fsub_rn(__int_as_float(d0), kMagic), f1 = __fsub_rn(__int_as_float(d1), kMagic);
  a0 = __fmaf_rn(__fmul_rn(f0, xs), ws, a0);
  a1 = __fmaf_rn(__fmul_rn(f1, xs), ws, a1);
}

// _mm512_reduce_add_ps over the 16 lane accumulators of a row, held by 8 consecutive threads (two each): lanes 8
// apart, 4 apart, 2 apart, then the last pair. Float addition is commutative, so which thread adds is free; the pairs
// are the tree's. The result is valid in the row's thread j = 0.
__device__ __forceinline__ float row_reduce(float a0, float a1) {
  a0 = __fadd_rn(a0, __shfl_down_sync(0xffffffffu, a0, 4, 8));
  a1 = __fadd_rn(a1, __shfl_down_sync(0xffffffffu, a1, 4, 8));
  a0 = __fadd_rn(a0, __shfl_down_sync(0xffffffffu, a0, 2, 8));
  a1 = __fadd_rn(a1, __shfl_down_sync(0xffffffffu, a1, 2, 8));
  a0 = __fadd_rn(a0, __shfl_down_sync(0xffffffffu, a0, 1, 8));
  a1 = __fadd_rn(a1, __shfl_down_sync(0xffffffffu, a1, 1, 8));
  return __fadd_rn(a0, a1);
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
  // The loops stay rolled: this runs once per CTA at the start of every launch, from a cold instruction cache, and
  // unrolled copies measured slower (decode step 2.38 ms rolled, 2.39 / 2.46 / 2.66 ms unrolled by 2 / 4 / 8).
  const int per = gs / 4, sub = lane & 3, g8 = (lane >> 2) & 7;
  const int groups = n / gs, slots = (groups + 7) / 8 * 32;  // 8 groups per warp-sized slot
  for (int t = tid; t < slots; t += kThreads) {
    const int grp = (t >> 5) * 8 + g8;
    const bool live = grp < groups;
    const float *xg = XF + grp * gs, *wg = NW + grp * gs;
    float mx = 0.0f;
    int bad = 0;
    if (live)
#pragma unroll 1
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
#pragma unroll 1
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
// The norm weights depend on no kernel: the caller stages them (stage_norm_weights) before waiting on the previous one.
__device__ __forceinline__ void stage_norm_weights(const GemvArgs &a, float *XF) {
  if (a.act == kActNormQuantize)
    stage_floats(XF + a.n, a.normw, a.n, false);
}

__device__ __forceinline__ void prepare_activation(const GemvArgs &a, int8_t *XQ, float *XS, float *XF, float *scratch,
                                                   int gs) {
  const int tid = threadIdx.x, n = a.n;
  const bool norm = a.act == kActNormQuantize;
  float *NW = XF + n;
  stage_floats(XF, a.xf, n, false);
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
  __syncthreads();  // this CTA's outputs are written
  // Acquire-release adds: each publishes the CTA's outputs (ordered before it by the barrier above) and, when it
  // completes a group, makes the other CTAs' rows of that group visible to the warp that quantizes it (ordered after
  // it by the barrier below).
  for (int i = tid; i < ng; i += kThreads) {
    const int g = g0 + i;
    const unsigned cnt = (unsigned)(min(r1, (g + 1) * gs) - max(r0, g * gs));
    unsigned before;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
                 : "=r"(before)
                 : "l"(kc_gemv_group_counter + g), "r"(cnt)
                 : "memory");
    flags[i] = before + cnt == (unsigned)gs;
  }
  __syncthreads();
  for (int i = warp; i < ng; i += kThreads / 32) {
    if (!flags[i])
      continue;
    const int g = g0 + i;
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
  // Whole octets of units per CTA (units < 2^31 / 1024, checked on the host).
  const int noct = (a.units + kOctRows - 1) / kOctRows;
  const int u0 = min(a.units, kOctRows * (int)((long long)noct * c / G));
  const int u1 = min(a.units, kOctRows * (int)((long long)noct * (c + 1) / G));
  if (u1 <= u0) {
    if (a.tail.kind && a.tail.kind != KC_TAIL_QUANTIZE_OUTPUT)  // the flag lives past the tail's scratch
      finish_tail(a, reinterpret_cast<float *>(smem), reinterpret_cast<int *>(smem + a.depth * a.stage_bytes));
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

  // Shared memory: the stages (1024-byte aligned for the swizzle), the control block, then the activations.
  uint8_t *stages = smem;
  uint8_t *ctrl = smem + depth * stage_bytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(ctrl);
  uint64_t *empty = full + kMaxDepth;
  volatile int *abort_flag = reinterpret_cast<int *>(ctrl + 16 * kMaxDepth);
  volatile int *issued = abort_flag + 1;
  int *tail_flag = const_cast<int *>(abort_flag) + 2;
  float *scratch = reinterpret_cast<float *>(ctrl + 16 * kMaxDepth + 16);
  float *XS = reinterpret_cast<float *>(ctrl + kCtrlBytes);
  int8_t *XQ = reinterpret_cast<int8_t *>(XS + ((n / gs + 3) & ~3));

  if (tid == 0) {
    for (int i = 0; i < depth; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kComputeWarps);
    }
    *abort_flag = 0;
    *issued = min(depth, S);
    fence_mbar_init();
  }
  __syncthreads();
  // Weights do not depend on the previous kernel: the first stage streams in before waiting for it. The others are
  // issued once the activation loads are on their way, so those few kilobytes do not queue behind the whole
  // prefetch on the way into this SM.
  if (warp == kComputeWarps && S > 0)
    issue_stage(m, gpc, a.kblock, subtile(plan, 0), 0, swiglu, lane, stages, &full[0]);
  stage_norm_weights(a, reinterpret_cast<float *>(XQ + ((n + 15) & ~15)));
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
    prepare_activation(a, XQ, XS, reinterpret_cast<float *>(XQ + ((n + 15) & ~15)), scratch, gs);
  }
  if (warp == kComputeWarps)
    for (int i = 1; i < depth && i < S; i++)
      issue_stage(m, gpc, a.kblock, subtile(plan, i / nchunks), i % nchunks, swiglu, lane, stages + i * stage_bytes,
                  &full[i]);
  __syncthreads();

  if (warp < kComputeWarps) {
    // ---- compute warps: warp w holds rows b, b+4, b+16, b+20 of each sub-tile (b = 8(w/4) + w%4), 8 threads each;
    // for SwiGLU rows 16.. are w3's, so a unit's w1 and w3 rows sit 16 lanes apart in one warp.
    const int rho = lane >> 3, j = lane & 7;
    const int pr = (warp >> 2) * 8 + (warp & 3) + (rho & 1) * 4 + (rho >> 1) * 16;
    const int r7 = pr & 7;
    const int unit_in_tile = swiglu ? (pr & 15) : pr;
    float a0 = 0.0f, a1 = 0.0f;
    int slot = 0, chunk = 0, sub = 0;
    unsigned phase = 0;
    for (int i = 0; i < S; i++) {
      if (!*abort_flag && !mbar_wait_bounded(&full[slot], phase))
        *abort_flag = 1;
      const uint8_t *buf = stages + slot * stage_bytes;
      const uint8_t *rowbuf = buf + (pr >> 3) * kOctBytes + r7 * kBoxCols;
      const float *wsr = reinterpret_cast<const float *>(buf + kWeightStage) + pr * gpc;
      const int8_t *xrow = XQ + chunk * kChunk;
      const float *xsc = XS + chunk * gpc;
      const int groups = min(gpc, (n - chunk * kChunk) / gs);
      if (GS == 64 && groups == kChunk / 64) {
#pragma unroll
        for (int h = 0; h < kChunk / 64; h += 4) {
          const float4 w4 = *reinterpret_cast<const float4 *>(wsr + h);
          const float4 x4 = *reinterpret_cast<const float4 *>(xsc + h);
          group_step<GS>(rowbuf, r7, xrow, h + 0, gs, j, x4.x, w4.x, a0, a1);
          group_step<GS>(rowbuf, r7, xrow, h + 1, gs, j, x4.y, w4.y, a0, a1);
          group_step<GS>(rowbuf, r7, xrow, h + 2, gs, j, x4.z, w4.z, a0, a1);
          group_step<GS>(rowbuf, r7, xrow, h + 3, gs, j, x4.w, w4.w, a0, a1);
        }
      } else {
        for (int g = 0; g < groups; g++)
          group_step<GS>(rowbuf, r7, xrow, g, gs, j, xsc[g], wsr[g], a0, a1);
      }
      // This warp's last read of the stage: release it to the producer.
      __syncwarp();
      if (lane == 0)
        mbar_arrive(&empty[slot]);
      if (chunk == nchunks - 1) {
        const Sub t = subtile(plan, sub);
        const float r = row_reduce(a0, a1);
        const float gate = __shfl_down_sync(0xffffffffu, r, 16);
        float *out = (t.seg == 0 ? out0 : t.seg == 1 ? out1 : out2) + t.row0;
        if (j == 0 && unit_in_tile < t.cnt) {
          if (swiglu) {
            if (rho < 2)
              out[unit_in_tile] = silu_gate_dev(r, gate);
          } else if (a.kind == KC_ADD) {
            out[unit_in_tile] = __fadd_rn(out[unit_in_tile], r);
          } else if (RED) {
            push_row(a.peer, par, seq, t.row0 + unit_in_tile, r);
          } else {
            out[unit_in_tile] = r;
          }
        }
        a0 = 0.0f, a1 = 0.0f;
      }
      if (++slot == depth)
        slot = 0, phase ^= 1u;
      if (++chunk == nchunks)
        chunk = 0, sub++;
    }
  } else {
    // ---- producer warp: refills stage slot i % depth with stage i once every compute warp has released stage
    // i - depth.
    int nchunk = depth % nchunks, nsub = depth / nchunks;  // chunk and sub-tile of stage i
    for (int i = depth; i < S; i++) {
      const int slot = i % depth;
      if (*abort_flag || !mbar_wait_bounded(&empty[slot], (unsigned)(i / depth - 1) & 1u)) {
        *abort_flag = 1;
        break;
      }
      issue_stage(m, gpc, a.kblock, subtile(plan, nsub), nchunk, swiglu, lane, stages + slot * stage_bytes,
                  &full[slot]);
      if (lane == 0)
        *issued = i + 1;
      if (++nchunk == nchunks)
        nchunk = 0, nsub++;
    }
  }
  // After an abort, let every copy still in flight land (bounded waits) before the shared memory goes away: for each
  // slot, the latest stage issued into it.
  __syncthreads();
  if (*abort_flag && tid == 0)
    for (int j = max(0, *issued - depth); j < *issued; j++)
      mbar_wait_bounded(&full[j % depth], (unsigned)(j / depth) & 1u);
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
    finish_tail(a, reinterpret_cast<float *>(stages), tail_flag);
  }
}


// The general rung, for shapes the TMA kernel does not take (group sizes that are not a power-of-two multiple of 64,
// scale rows that are not 16-byte multiples, unaligned pointers): one warp per output row, in the order the
// reference's k_matmul_q8 uses for the group size (q8_dots, src/gemv.c:401-438):
//  - gs % 64 == 0: the AVX-512 lane order of dots_q8_body, lanes 0-15 of the warp being the 16 vector lanes (bitwise
//    the TMA kernel);
//  - otherwise its portable loop: the exact int32 group dot (reduced across the warp), then, by lane 0,
//    val = val + ((float)dot * ws[g]) * xs[g], no fused multiply-add.
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
  const bool avx = gs % 64 == 0;
  float acc[2] = {0.0f, 0.0f};
  for (int pass = 0; pass < (kind == KC_SWIGLU ? 2 : 1); pass++) {
    const int8_t *w = pass ? w3q + row * ld : wq;
    const float *sc = pass ? w3s + row * (ld / gs) : ws;
    float a = 0.0f;
    for (int g = 0; g < n / gs; g++) {
      int dot = 0;
      if (avx) {
        if (lane < 16)
          for (int c = 0; c < gs; c += 64)
            for (int k = 0; k < 4; k++)
              dot += (int)xq[g * gs + c + 4 * lane + k] * (int)w[g * gs + c + 4 * lane + k];
        a = __fmaf_rn(__fmul_rn(__int2float_rn(dot), xs[g]), sc[g], a);
      } else {
        for (int k = lane; k < gs; k += 32)
          dot += (int)xq[g * gs + k] * (int)w[g * gs + k];
#pragma unroll
        for (int o = 16; o; o >>= 1)
          dot += __shfl_xor_sync(0xffffffffu, dot, o);
        a = __fadd_rn(a, __fmul_rn(__fmul_rn(__int2float_rn(dot), sc[g]), xs[g]));
      }
    }
    if (avx) {  // _mm512_reduce_add_ps: lanes 8 apart, 4, 2, 1
#pragma unroll
      for (int o = 8; o; o >>= 1)
        a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, o, 16));
    }
    acc[pass] = a;
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
  return (size_t)depth * stage_bytes + kCtrlBytes + (size_t)((n / gs + 3) & ~3) * 4 + (size_t)((n + 15) & ~15) +
         (size_t)act_floats * 4 + 1024;
}

// The weight map moves octets of rows ([8 K-blocks x 8 rows x 128 B] boxes, or [128 B x 8 rows] without k-block
// maps); the scale map moves [gpc floats x scale_rows] boxes.
bool encode_weight(CUtensorMap *wmap, CUtensorMap *smap, const int8_t *wq, const float *ws, int rows, int n,
                   long long ld, int gs, int scale_rows, bool kblock) {
  const int gpc = kChunk / gs;
  bool ok = kblock ? kc_tmap_kblocks(wmap, wq, (uint64_t)n, (uint64_t)rows, (uint64_t)ld, kBoxes, kOctRows)
                   : kc_tmap_2d(wmap, wq, 1, (uint64_t)n, (uint64_t)rows, (uint64_t)ld, kBoxCols, kOctRows, true);
  return ok &&
         kc_tmap_2d(smap, ws, 4, (uint64_t)(n / gs), (uint64_t)rows, (uint64_t)(ld / gs) * 4, gpc, scale_rows, false);
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
  // The lane order is the reference's for gs % 64 == 0; other group sizes take the general rung's portable order.
  if (gs < 64 || gs > kChunk || (gs & (gs - 1)) || n % gs || ld % gs || ld < n || ((ld / gs) * 4) % 16 ||
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
  const int scale_rows = swiglu ? kTileRows / 2 : kTileRows;
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
      ok = encode_weight(&M.wmap[s], &M.smap[s], segs[s].wq, segs[s].ws, segs[s].d, n, ld, gs, scale_rows, kblock) &&
           (!swiglu ||
            encode_weight(&M.w3map, &M.s3map, segs[s].w3q, segs[s].w3s, segs[s].d, n, ld, gs, scale_rows, kblock));
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
#define KC_GEMV_MAX_DEPTH 5
#endif
  static_assert(KC_GEMV_MAX_DEPTH <= kMaxDepth, "pipeline depth");
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
  const int octets = (units + kOctRows - 1) / kOctRows;  // the CTAs split the units in whole octets
  int grid = octets < sms ? octets : sms;
  // The launch ends with its slowest CTA: when the octets do not divide evenly over every SM, the largest CTA count
  // from 3/4 of the SMs up that divides them gives every CTA the same work (1792 octets: 128 CTAs of 14 instead of
  // 16 of 13 and 132 of 12; the weight stream is HBM-bound, so fewer CTAs lose no bandwidth).
  if (grid == sms && octets % sms)
    for (int g = sms - 1; g >= sms - sms / 4; g--)
      if (octets % g == 0) {
        grid = g;
        break;
      }
  if (grid_limit > 0 && grid > grid_limit)
    grid = grid_limit;
  if (kind == KC_REDUCE_ADD)  // one grid size for every call: each CTA's counter counts every call
    grid = sms < kPeerGemvMaxCtas ? sms : kPeerGemvMaxCtas;
  const int variant = (gs == 64 ? 0 : 1) + (kind == KC_REDUCE_ADD ? 2 : 0);
  void (*const kernels[4])(const GemvMaps, const GemvArgs) = {gemv_q8_kernel<64, false>, gemv_q8_kernel<0, false>,
                                                              gemv_q8_kernel<64, true>, gemv_q8_kernel<0, true>};
  if (kc_allow_smem(reinterpret_cast<const void *>(kernels[variant]), 227 * 1024) != cudaSuccess)
    return -2;
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

