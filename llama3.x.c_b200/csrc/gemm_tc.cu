// Q8_0 W8A8 prefill GEMM for sm_100a on the 5th-generation tensor core:
//   C[m][n] (op)= sum over 64-groups g of (float)dot_g(xq[m], wq[n]) * xs[m][g] * ws[n][g]
// with the epilogues of the reference's batched GEMM (q8_gemm_chunks, src/gemm.c:963-989: STORE / ADD / PARTIAL, and
// SWIGLU on a w1/w3 pair) over 1-3 segments that share the activations (k_gemm_q8, include/gemm.h:130-133).
//
// Arithmetic, bitwise the reference's AMX-INT8 backend (amx_q8_chunk, src/gemm.c:564-608) and this library's GEMV:
// every group dot is an exact int32 (tcgen05.mma kind::i8, two K=32 steps per 64-group), and every output rescales
// the groups in ascending order as acc = fmaf((float)dot * xs, ws, acc) from acc = 0.
//
// Tiling: the MMA's M side is 128 weight rows (for SwiGLU 64 w1 and 64 w3 rows, interleaved in 16-row blocks so
// that the two halves of an output sit in lanes L and L+16 of one warp), its N side 128 tokens; a persistent CTA per
// SM walks its tiles (tokens fastest, so the CTAs running together share weight stripes in L2).
//   warp 0      TMA producer: per stage (two groups, 128 B of K) one [128 x 128 B] weight box (eight 16-row boxes
//               for SwiGLU) and one [128 x 128 B] activation box, both 128B-swizzled (the canonical K-major UMMA
//               layout), into a ring of 6 stages the MMA releases; and the stage's transposed activation scales
//               [2 groups x 128 tokens] into a ring of 8 the epilogue releases.
//   warp 1      MMA issuer: allocates 512 TMEM columns (four 128 x 128 int32 buffers), issues two MMAs per group into
//               the next buffer the epilogue has released, commits the buffer to the epilogue and the stage to the ring.
//   warps 2-17  epilogue (warp % 4 = TMEM lane quadrant = 32 weight rows, (warp - 2) / 4 = 32-token column
//               quarter): per group one read of its 32 x 32 int32 dots as packed column pairs, the buffer released as
//               soon as they are in registers, then the promotion with packed f32x2 instructions; four epilogue warps
//               per SM sub-partition cover one another's TMEM read latency. Four buffers let the MMA run up to three
//               groups ahead of the promotion. 16-column chunks past the last token are not promoted (they are never
//               stored). Weight scales are read four groups at a time, the next four a step ahead.
// Group promotion: the group's first MMA overwrites its TMEM buffer (no clearing), the epilogue converts each exact
// int32 dot to float (exact: |dot| <= 64*128^2 < 2^24) and applies mul, fma as packed pairs.
//
// Every mbarrier wait is bounded (a timeout raises KC_ERR_TIMEOUT, sets a CTA abort flag that turns the remaining
// waits into no-ops, and the CTA still releases its TMEM).
#include <cuda.h>
#include <stdio.h>
#include <string.h>

#include "common.cuh"
#include "kernels_cuda_internal.h"
#include "tcgen05.cuh"
#include "tmap.h"

namespace {

constexpr int kTM = 128;                      // weight rows per tile (MMA M)
constexpr int kTN = 128;                      // tokens per tile (MMA N)
constexpr int kStages = 6;                    // operand ring (released by the MMA)
constexpr int kXsStages = 8;                  // activation-scale ring (released by the epilogue)
constexpr int kStageA = kTM * 128;            // weights: 128 rows x 128 B
constexpr int kStageB = kTN * 128;            // activations: 128 tokens x 128 B
constexpr int kStageBytes = kStageA + kStageB;
constexpr int kStageX = 2 * kTN * 4;          // activation scales of one stage: 2 groups x 128 tokens
constexpr int kEpiWarp0 = 2;                  // warps 0 (TMA) and 1 (MMA) come first
constexpr int kEpiCols = 32;                  // token columns per epilogue thread
constexpr int kEpiWarps = 4 * (kTN / kEpiCols);  // 4 lane quadrants x 4 column quarters
constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;
constexpr int kTmemBufs = 4;                  // 128-column int32 accumulators in flight
constexpr int kTmemCols = kTmemBufs * 128;
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + kXsStages * kStageX + 512 + 1024;

struct __align__(64) GemmMaps {
  CUtensorMap w[3];  // weights per segment: boxes [128 B x 128 rows]; SwiGLU w1: [128 B x 16 rows]
  CUtensorMap w3;    // SwiGLU w3: [128 B x 16 rows]
  CUtensorMap x;     // activations [M][K]: boxes [128 B x 128 tokens]
  CUtensorMap xs;    // transposed activation scales [groups][ldt]: boxes [128 tokens x 2 groups]
};

struct GemmSegDev {
  float *c;
  const float *ws;
  const float *ws3;
  int ldc, n, kind, tile0;
};

struct GemmArgs {
  GemmSegDev seg[3];
  int nseg;
  int M, K, groups, stages_per_tile, m_tiles, total_tiles;
  int32_t *dots;  // test hook: raw group dots of segment 0, [g][M][n]
};

struct Tile {
  int s, n0, m0;
  bool swiglu;
};

__device__ __forceinline__ Tile decode_tile(const GemmArgs &a, int t) {
  Tile r;
  r.s = (a.nseg > 1 && t >= a.seg[1].tile0) ? 1 : 0;
  if (a.nseg > 2 && t >= a.seg[2].tile0)
    r.s = 2;
  const int tile0 = r.s == 0 ? a.seg[0].tile0 : r.s == 1 ? a.seg[1].tile0 : a.seg[2].tile0;
  const int kind = r.s == 0 ? a.seg[0].kind : r.s == 1 ? a.seg[1].kind : a.seg[2].kind;
  r.swiglu = kind == KC_SWIGLU;
  const int local = t - tile0;
  const int nt = local / a.m_tiles;
  r.m0 = (local - nt * a.m_tiles) * kTN;
  r.n0 = nt * (r.swiglu ? kTM / 2 : kTM);
  return r;
}

__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, unsigned parity, volatile int *abort_flag) {
  if (*abort_flag)
    return false;
  if (mbar_wait_sleep_bounded(bar, parity))
    return true;
  *abort_flag = 1;
  return false;
}

// A packed pair of exact int32 group dots as the packed pair of floats, each half converted exactly
// (|dot| <= 64 * 128^2 = 2^20 < 2^24).
__device__ __forceinline__ uint64_t dots_to_f2(uint64_t v) {
  uint64_t r;
  asm("{\n\t.reg .b32 lo, hi;\n\t.reg .f32 flo, fhi;\n\t"
      "mov.b64 {lo, hi}, %1;\n\t"
      "cvt.rn.f32.s32 flo, lo;\n\tcvt.rn.f32.s32 fhi, hi;\n\t"
      "mov.b64 %0, {flo, fhi};\n\t}"
      : "=l"(r)
      : "l"(v));
  return r;
}

// Promotes 16 token columns of one group, held as 8 packed pairs: acc[p] = fma(((float)dot) * xs, ws, acc[p]) (the
// reference's rounding sequence: one rounded product, then one fused multiply-add). xs: the 16 activation scales.
__device__ __forceinline__ void promote16(uint64_t *acc, const uint64_t *r, const float *xs, uint64_t ws2) {
  const ulonglong2 *xs2 = reinterpret_cast<const ulonglong2 *>(xs);
#pragma unroll
  for (int p4 = 0; p4 < 4; p4++) {
    const ulonglong2 x = xs2[p4];
    acc[2 * p4] = f2_fma(f2_mul(dots_to_f2(r[2 * p4]), x.x), ws2, acc[2 * p4]);
    acc[2 * p4 + 1] = f2_fma(f2_mul(dots_to_f2(r[2 * p4 + 1]), x.y), ws2, acc[2 * p4 + 1]);
  }
}

// DOTS: the test hook's variant, which stores the raw int32 group dots instead of promoting.
template <bool DOTS>
__global__ void __launch_bounds__(kThreads, 1) gemm_q8_tc_kernel(const __grid_constant__ GemmMaps mp, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  // The 128-byte swizzle is a function of the address bits, so the operand stages start on a 1024-byte boundary.
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t *stages = smem;
  float *xsring = reinterpret_cast<float *>(smem + kStages * kStageBytes);
  uint8_t *tail = smem + kStages * kStageBytes + kXsStages * kStageX;
  uint64_t *full = reinterpret_cast<uint64_t *>(tail);
  uint64_t *empty = full + kStages;
  uint64_t *xfull = empty + kStages;
  uint64_t *xempty = xfull + kXsStages;
  uint64_t *tfull = xempty + kXsStages;
  uint64_t *tempty = tfull + kTmemBufs;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + kTmemBufs);
  volatile int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < kXsStages; i++) {
      mbar_init(&xfull[i], 1);
      mbar_init(&xempty[i], kEpiWarps);
    }
    for (int i = 0; i < kTmemBufs; i++) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1)
    tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();

  const int G = gridDim.x;
  const int spt = a.stages_per_tile, groups = a.groups;

  if (warp == 0) {
    // ---- TMA producer (the whole warp loops and waits, so no lane idles at the CTA barrier; lane 0 issues) ----
    int st = 0;
    for (int t = blockIdx.x; t < a.total_tiles; t += G) {
      const Tile tl = decode_tile(a, t);
      for (int j = 0; j < spt; j++, st++) {
        const int slot = st % kStages, use = st / kStages;
        const int xslot = st % kXsStages, xuse = st / kXsStages;
        if (!wait_or_abort(&empty[slot], (use & 1) ^ 1, abort_flag) ||
            !wait_or_abort(&xempty[xslot], (xuse & 1) ^ 1, abort_flag))
          continue;
        uint8_t *base = stages + slot * kStageBytes;
        if (lane != 0)
          continue;
        mbar_arrive_expect_tx(&full[slot], kStageBytes);
        mbar_arrive_expect_tx(&xfull[xslot], kStageX);
        const int k0 = j * 128;
        if (tl.swiglu) {
          // Rows 32i .. 32i+15 of the tile are w1 rows n0+16i .., rows 32i+16 .. 32i+31 the matching w3 rows, so
          // lanes L and L+16 of every epilogue warp hold the two halves of one SwiGLU output.
#pragma unroll
          for (int i = 0; i < 4; i++) {
            tma_load_2d(base + (32 * i) * 128, &mp.w[0], k0, tl.n0 + 16 * i, &full[slot]);
            tma_load_2d(base + (32 * i + 16) * 128, &mp.w3, k0, tl.n0 + 16 * i, &full[slot]);
          }
        } else {
          tma_load_2d(base, &mp.w[0] + tl.s, k0, tl.n0, &full[slot]);
        }
        tma_load_2d(base + kStageA, &mp.x, k0, tl.m0, &full[slot]);
        tma_load_2d(xsring + xslot * (kStageX / 4), &mp.xs, tl.m0, 2 * j, &xfull[xslot]);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer (the whole warp loops and waits; lane 0 issues the MMAs and commits) ----
    const uint32_t idesc = umma_idesc_i8(kTM, kTN);
    int st = 0, gidx = 0;
    for (int t = blockIdx.x; t < a.total_tiles; t += G) {
      for (int j = 0; j < spt; j++, st++) {
        const int slot = st % kStages, use = st / kStages;
        const bool have = wait_or_abort(&full[slot], use & 1, abort_flag);
        tc_fence_after();
        const uint8_t *base = stages + slot * kStageBytes;
        const uint64_t adesc = umma_desc_sw128(base), bdesc = umma_desc_sw128(base + kStageA);
        for (int gg = 0; gg < 2 && 2 * j + gg < groups; gg++, gidx++) {
          const int b = gidx % kTmemBufs, ub = gidx / kTmemBufs;
          // A fresh barrier's preceding phase counts as complete, so the first use of each buffer does not wait.
          const bool ok = wait_or_abort(&tempty[b], (ub & 1) ^ 1, abort_flag) && have;
          tc_fence_after();
          if (ok && lane == 0) {
            // The group's first K step overwrites the buffer, the second accumulates onto it.
#pragma unroll
            for (int k = 0; k < 2; k++) {
              const uint64_t off = (uint64_t)((gg * 64 + k * 32) >> 4);
              umma_i8(tmem + b * kTN, adesc + off, bdesc + off, idesc, k > 0);
            }
          }
          if (lane == 0)
            umma_commit(&tfull[b]);
          __syncwarp();
        }
        if (lane == 0)
          umma_commit(&empty[slot]);
        __syncwarp();
      }
    }
  } else if (warp >= kEpiWarp0) {
    // ---- epilogue: promotion of every group, in order ----
    const int q = warp & 3, h = (warp - kEpiWarp0) >> 2;  // lane quadrant, 32-token column quarter
    const int row = 32 * q + lane;  // TMEM lane = row of the weight tile
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + kEpiCols * h;
    int st = 0, gidx = 0;
    for (int t = blockIdx.x; t < a.total_tiles; t += G) {
      const Tile tl = decode_tile(a, t);
      // Scalars of this tile's segment (selected field by field: a whole-struct select would go to local memory).
      const int seg_n = tl.s == 0 ? a.seg[0].n : tl.s == 1 ? a.seg[1].n : a.seg[2].n;
      const int seg_ldc = tl.s == 0 ? a.seg[0].ldc : tl.s == 1 ? a.seg[1].ldc : a.seg[2].ldc;
      const int seg_kind = tl.s == 0 ? a.seg[0].kind : tl.s == 1 ? a.seg[1].kind : a.seg[2].kind;
      float *const seg_c = tl.s == 0 ? a.seg[0].c : tl.s == 1 ? a.seg[1].c : a.seg[2].c;
      const float *const seg_ws = tl.s == 0 ? a.seg[0].ws : tl.s == 1 ? a.seg[1].ws : a.seg[2].ws;
      const bool w3row = tl.swiglu && lane >= 16;
      const int n = tl.n0 + (tl.swiglu ? 16 * q + (lane & 15) : row);
      const bool row_ok = n < seg_n;
      const float *wsr = (w3row ? a.seg[0].ws3 : seg_ws) + (size_t)min(n, seg_n - 1) * groups;
      // Token columns of this warp that hold activation rows (warp-uniform). 16-column chunks at or past it are
      // never stored, so their promotion is skipped: with few tokens the epilogue does only the columns it writes.
      const int live = a.M - (tl.m0 + kEpiCols * h);
      uint64_t acc[kEpiCols / 2];
#pragma unroll
      for (int i = 0; i < kEpiCols / 2; i++)
        acc[i] = 0;
      // Per group: one read of the warp's 32 columns, the buffer released as soon as they are in registers, then the
      // promotion (the other epilogue warps of the sub-partition cover the read's latency). Weight scales come four
      // groups at a time, the next four loaded a step ahead.
      const float4 *ws4 = reinterpret_cast<const float4 *>(wsr);
      float4 wq4 = __ldg(ws4), wn4 = groups > 4 ? __ldg(ws4 + 1) : wq4;
      for (int j = 0; j < spt; j++, st++) {
        const int xslot = st % kXsStages;
        wait_or_abort(&xfull[xslot], (st / kXsStages) & 1, abort_flag);
        const float *xsT = xsring + xslot * (kStageX / 4);
        if (j > 0 && (j & 1) == 0) {  // groups 2j, 2j + 1 start a new four
          wq4 = wn4;
          if (2 * j + 4 < groups)
            wn4 = __ldg(ws4 + (j >> 1) + 1);
        }
#pragma unroll
        for (int gg = 0; gg < 2; gg++, gidx++) {
          const int g = 2 * j + gg, b = gidx % kTmemBufs;
          const bool ok = wait_or_abort(&tfull[b], (gidx / kTmemBufs) & 1, abort_flag);
          tc_fence_after();
          uint64_t r[16];
          tmem_ld32_pairs(tq + b * kTN, r);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0)
            mbar_arrive(&tempty[b]);
          if (!ok)
            continue;
          if (DOTS) {
            if (row_ok && tl.s == 0 && !tl.swiglu)
#pragma unroll
              for (int i = 0; i < 32; i++)
                if (tl.m0 + kEpiCols * h + i < a.M)
                  a.dots[((size_t)g * a.M + tl.m0 + kEpiCols * h + i) * seg_n + n] =
                      (int32_t)(uint32_t)(r[i >> 1] >> (32 * (i & 1)));
            continue;
          }
          const float wv = (j & 1) ? (gg ? wq4.w : wq4.z) : (gg ? wq4.y : wq4.x);
          const uint64_t ws2 = f2_pack(wv, wv);
          const float *xs = xsT + gg * kTN + kEpiCols * h;
          if (live > 0)
            promote16(acc, r, xs, ws2);
          if (live > 16)
            promote16(acc + 8, r + 8, xs + 16, ws2);
        }
        __syncwarp();
        if (lane == 0)
          mbar_arrive(&xempty[xslot]);
      }
      if (DOTS)
        continue;
      // ---- write the tile: thread = weight row n, 64 tokens ----
      const int mbase = tl.m0 + kEpiCols * h;
      if (tl.swiglu) {
#pragma unroll
        for (int i = 0; i < kEpiCols / 2; i++) {
          float lo, hi, glo, ghi;
          f2_unpack(acc[i], lo, hi);
          glo = __shfl_down_sync(0xffffffffu, lo, 16);
          ghi = __shfl_down_sync(0xffffffffu, hi, 16);
          const int m = mbase + 2 * i;
          if (!w3row && row_ok) {
            if (m < a.M)
              seg_c[(size_t)m * seg_ldc + n] = silu_gate_dev(lo, glo);
            if (m + 1 < a.M)
              seg_c[(size_t)(m + 1) * seg_ldc + n] = silu_gate_dev(hi, ghi);
          }
        }
      } else if (row_ok) {
#pragma unroll
        for (int i = 0; i < kEpiCols / 2; i++) {
          float lo, hi;
          f2_unpack(acc[i], lo, hi);
          const int m = mbase + 2 * i;
          float *c0 = seg_c + (size_t)m * seg_ldc + n;
          if (m < a.M)
            *c0 = seg_kind == KC_ADD ? __fadd_rn(*c0, lo) : lo;
          if (m + 1 < a.M)
            c0[seg_ldc] = seg_kind == KC_ADD ? __fadd_rn(c0[seg_ldc], hi) : hi;
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// xs [M][groups] -> xsT [groups][ldt] (ldt >= M, a multiple of 4 so the TMA row stride is 16-byte aligned).
__global__ void transpose_scales_kernel(float *xsT, const float *xs, int M, int groups, int ldt) {
  pdl_wait();
  pdl_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= groups * ldt)
    return;
  const int g = i / ldt, m = i - g * ldt;
  xsT[i] = m < M ? xs[(size_t)m * groups + g] : 0.0f;
}

}  // namespace

size_t kc_gemm_xst_floats(int M, int groups) { return (size_t)groups * (size_t)((M + 3) & ~3); }

int kc_launch_transpose_scales(float *xsT, const float *xs, int M, int groups, cudaStream_t stream) {
  const int ldt = (M + 3) & ~3;
  const long long total = (long long)groups * ldt;
  if (total == 0)
    return 0;
  kc_launch_pdl(transpose_scales_kernel, (unsigned)((total + 255) / 256), 256, 0, stream, xsT, xs, M, groups, ldt);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

bool kc_gemm_tc_supported(const KcGemmSeg *segs, int nseg, const int8_t *xq, int M, int K, int gs) {
  if (gs != 64 || K <= 0 || K % 256 || M <= 0 || ((uintptr_t)xq & 15))
    return false;
  for (int s = 0; s < nseg; s++) {
    if (((uintptr_t)segs[s].wq & 15) || ((uintptr_t)segs[s].ws & 15))
      return false;
    if (segs[s].kind == KC_SWIGLU && (((uintptr_t)segs[s].w3q & 15) || ((uintptr_t)segs[s].w3s & 15)))
      return false;
  }
  return true;
}

// xsT: transposed activation scales [K/64][round_up(M, 4)] (kc_launch_transpose_scales). dots: test hook or NULL.
int kc_launch_gemm_tc(const KcGemmSeg *segs, int nseg, const int8_t *xq, const float *xsT, int M, int K,
                      int32_t *dots, cudaStream_t stream) {
  thread_local GemmMaps mp;
  GemmArgs a;
  memset(&mp, 0, sizeof(mp));
  memset(&a, 0, sizeof(a));
  const int groups = K / 64, ldt = (M + 3) & ~3;
  a.nseg = nseg;
  a.M = M;
  a.K = K;
  a.groups = groups;
  a.stages_per_tile = (groups + 1) / 2;
  a.m_tiles = (M + kTN - 1) / kTN;
  a.dots = dots;
  int tiles = 0;
  for (int s = 0; s < nseg; s++) {
    const bool swiglu = segs[s].kind == KC_SWIGLU;
    const int rows_per_tile = swiglu ? kTM / 2 : kTM;
    a.seg[s].c = segs[s].c;
    a.seg[s].ws = segs[s].ws;
    a.seg[s].ws3 = segs[s].w3s;
    a.seg[s].ldc = segs[s].ldc;
    a.seg[s].n = segs[s].n;
    a.seg[s].kind = segs[s].kind;
    a.seg[s].tile0 = tiles;
    if (segs[s].n <= 0)
      continue;
    tiles += ((segs[s].n + rows_per_tile - 1) / rows_per_tile) * a.m_tiles;
    if (swiglu) {
      if (s != 0 || nseg != 1)
        return -1;  // the SwiGLU pair is a segment of its own (the reference's engine issues it alone)
      if (!kc_tmap_2d(&mp.w[0], segs[s].wq, 1, K, segs[s].n, K, 128, 16, true) ||
          !kc_tmap_2d(&mp.w3, segs[s].w3q, 1, K, segs[s].n, K, 128, 16, true))
        return -1;
    } else if (!kc_tmap_2d(&mp.w[s], segs[s].wq, 1, K, segs[s].n, K, 128, kTM, true)) {
      return -1;
    }
  }
  a.total_tiles = tiles;
  if (tiles == 0)
    return 0;
  if (!kc_tmap_2d(&mp.x, xq, 1, K, M, K, 128, kTN, true) ||
      !kc_tmap_2d(&mp.xs, xsT, 4, ldt, groups, (uint64_t)ldt * 4, kTN, 2, false))
    return -1;
  const size_t smem = kSmemBytes;
  auto kern = dots ? gemm_q8_tc_kernel<true> : gemm_q8_tc_kernel<false>;
  if (kc_allow_smem(reinterpret_cast<const void *>(kern), (int)smem) != cudaSuccess)
    return -2;
  const int sms = kc_device_sms();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles < sms ? tiles : sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = kc_pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mp, a);
  if (e != cudaSuccess) {
    cudaFuncAttributes fa;
    cudaFuncGetAttributes(&fa, kern);
    fprintf(stderr, "gemm_q8_tc_kernel launch: %s (regs %d, threads %d, max threads %d, smem %zu + static %zu)\n",
            cudaGetErrorString(e), fa.numRegs, kThreads, fa.maxThreadsPerBlock, smem, fa.sharedSizeBytes);
    return -2;
  }
  return 0;
}
