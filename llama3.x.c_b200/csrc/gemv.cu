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
// q8_team_static, src/gemv.c:483-490), walks it in sub-tiles of 32 physical weight rows, and streams each sub-tile
// through shared memory in 1 KiB K-chunks with 1-D bulk copies (the TMA unit, one copy per row, completing on an
// mbarrier), several stages deep. Inside a stage, lane r of every warp owns weight row r, and warp w takes groups
// w, w+8, ... of the chunk, so the int32 dots need no shuffles; warp 0 then runs the ordered fp32 chain for all 32
// rows (one lane per row) from a small transposed buffer. Rows in shared memory are padded by 16 bytes so the 16-byte
// loads of 8 consecutive lanes hit distinct banks.
#include "common.cuh"
#include "kernels_cuda_internal.h"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTileRows = 32;  // physical weight rows per sub-tile (one per lane)
constexpr int kPad = 16;
constexpr int kMaxGroupsPerChunk = 32;

struct GemvSegDev {
  float *out;
  const int8_t *wq;
  const float *ws;
  const int8_t *w3q;
  const float *w3s;
  int d;
  int unit0;
};

struct GemvArgs {
  GemvSegDev seg[3];
  int nseg;
  const int8_t *xq;
  const float *xs;
  int n;          // inputs (K)
  long long ld;   // weight row stride in values (multiple of gs)
  int gs;
  int kind;       // KC_STORE / KC_ADD / KC_PARTIAL / KC_SWIGLU
  int units;      // output rows over all segments
  int kc;         // bytes per K-chunk
  int nchunks;
  int depth;      // pipeline stages
  int ws_vec4;    // weight-scale rows are 16-byte aligned: load them as float4
};

struct RowRef {
  const int8_t *wq;
  const float *ws;
  float *out;
  int local;
};

__device__ __forceinline__ RowRef row_of(const GemvArgs &a, int unit, bool second) {
  int s = 0;
  if (a.nseg > 1 && unit >= a.seg[1].unit0)
    s = 1;
  if (a.nseg > 2 && unit >= a.seg[2].unit0)
    s = 2;
  const GemvSegDev &g = a.seg[s];
  RowRef r;
  r.local = unit - g.unit0;
  r.out = g.out;
  r.wq = (second ? g.w3q : g.wq) + (long long)r.local * a.ld;
  r.ws = (second ? g.w3s : g.ws) + (long long)r.local * (a.ld / a.gs);
  return r;
}

struct StageInfo {
  int ub;      // first unit of the sub-tile
  int cnt;     // units in the sub-tile
  int chunk;   // K-chunk index
  int bytes;   // bytes of this chunk per row
};

__device__ __forceinline__ StageInfo stage_info(const GemvArgs &a, int u0, int u1, int tile_units, int i) {
  StageInfo s;
  int sub = i / a.nchunks;
  s.chunk = i - sub * a.nchunks;
  s.ub = u0 + sub * tile_units;
  s.cnt = min(tile_units, u1 - s.ub);
  s.bytes = min(a.kc, a.n - s.chunk * a.kc);
  return s;
}

__device__ __forceinline__ bool lane_active(bool swiglu, int lane, int cnt) {
  return swiglu ? (lane & 15) < cnt : lane < cnt;
}

// Issued by all 32 lanes of one warp: lane r copies physical row r of the stage.
__device__ __forceinline__ void issue_stage(const GemvArgs &a, const StageInfo &s, bool swiglu, int lane,
                                            uint8_t *buf, uint64_t *bar) {
  int rows = swiglu ? 2 * s.cnt : s.cnt;
  if (lane == 0)
    mbar_arrive_expect_tx(bar, (unsigned)(rows * s.bytes));
  __syncwarp();
  if (lane_active(swiglu, lane, s.cnt)) {
    int unit = s.ub + (swiglu ? (lane & 15) : lane);
    RowRef r = row_of(a, unit, swiglu && lane >= 16);
    bulk_g2s(buf + lane * (a.kc + kPad), r.wq + (long long)s.chunk * a.kc, (unsigned)s.bytes, bar);
  }
}

__device__ __forceinline__ void load_scales(const GemvArgs &a, const StageInfo &s, bool swiglu, int lane,
                                            float (&w)[kMaxGroupsPerChunk]) {
  if (!lane_active(swiglu, lane, s.cnt))
    return;
  int unit = s.ub + (swiglu ? (lane & 15) : lane);
  RowRef r = row_of(a, unit, swiglu && lane >= 16);
  int gpc = a.kc / a.gs, g0 = s.chunk * gpc, groups = s.bytes / a.gs;
  const float *p = r.ws + g0;
  if (a.ws_vec4 && (groups & 3) == 0) {
#pragma unroll
    for (int g = 0; g < kMaxGroupsPerChunk; g += 4)
      if (g < groups) {
        float4 v = __ldg(reinterpret_cast<const float4 *>(p + g));
        w[g] = v.x, w[g + 1] = v.y, w[g + 2] = v.z, w[g + 3] = v.w;
      }
  } else {
#pragma unroll
    for (int g = 0; g < kMaxGroupsPerChunk; g++)
      if (g < groups)
        w[g] = __ldg(p + g);
  }
}

__global__ void __launch_bounds__(kThreads, 1) gemv_q8_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const bool swiglu = a.kind == KC_SWIGLU;
  const int tile_units = swiglu ? kTileRows / 2 : kTileRows;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, c = blockIdx.x;
  const int u0 = (int)((long long)a.units * c / G), u1 = (int)((long long)a.units * (c + 1) / G);
  if (u1 <= u0)
    return;
  const int nsub = (u1 - u0 + tile_units - 1) / tile_units;
  const int S = nsub * a.nchunks;
  const int gpc = a.kc / a.gs;
  const int row_bytes = a.kc + kPad;

  // Carve shared memory: barriers, abort flag, activation scales, activations, the chain buffer, the stages.
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
  int *abort_flag = reinterpret_cast<int *>(smem + 8 * 16);
  float *XS = reinterpret_cast<float *>(smem + 256);
  int8_t *XQ = reinterpret_cast<int8_t *>(smem + 256 + ((a.n / a.gs * 4 + 15) & ~15));
  float *T = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(XQ) + ((a.n + 15) & ~15));
  uint8_t *stages = reinterpret_cast<uint8_t *>(T) + 2 * kMaxGroupsPerChunk * kTileRows * 4;

  if (tid == 0) {
    for (int i = 0; i < a.depth; i++)
      mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0)
    for (int i = 0; i < a.depth && i < S; i++)
      issue_stage(a, stage_info(a, u0, u1, tile_units, i), swiglu, lane, stages + i * kTileRows * row_bytes,
                  &bars[i]);
  // Activations (quantized) and their scales, once per CTA.
  for (int i = tid; i < a.n / 16; i += kThreads)
    reinterpret_cast<int4 *>(XQ)[i] = __ldg(reinterpret_cast<const int4 *>(a.xq) + i);
  for (int i = tid; i < a.n / a.gs; i += kThreads)
    XS[i] = __ldg(a.xs + i);

  float wcur[kMaxGroupsPerChunk], wnext[kMaxGroupsPerChunk];
  float acc = 0.0f;
  int aborted_at = -1;
  if (warp == 0)
    load_scales(a, stage_info(a, u0, u1, tile_units, 0), swiglu, lane, wcur);
  __syncthreads();

  for (int i = 0; i < S; i++) {
    const int slot = i % a.depth;
    const StageInfo s = stage_info(a, u0, u1, tile_units, i);
    if (warp == 0 && i + 1 < S)
      load_scales(a, stage_info(a, u0, u1, tile_units, i + 1), swiglu, lane, wnext);
    if (!mbar_wait_bounded(&bars[slot], (unsigned)(i / a.depth) & 1u))
      *abort_flag = 1;
    const uint8_t *buf = stages + slot * kTileRows * row_bytes;
    float *Tb = T + (i & 1) * kMaxGroupsPerChunk * kTileRows;
    const int groups = s.bytes / a.gs;
    if (lane_active(swiglu, lane, s.cnt)) {
      const uint8_t *wrow = buf + lane * row_bytes;
      const int8_t *xrow = XQ + s.chunk * a.kc;
      for (int g = warp; g < groups; g += kWarps) {
        int dot = 0;
        for (int q = 0; q < a.gs; q += 16)
          dot = dot16(lds128(wrow + g * a.gs + q), lds128(xrow + g * a.gs + q), dot);
        Tb[g * kTileRows + lane] = __fmul_rn(__int2float_rn(dot), XS[s.chunk * gpc + g]);
      }
    }
    __syncthreads();
    if (*abort_flag) {
      aborted_at = i;
      break;
    }
    if (warp == 0) {
      if (i + a.depth < S)
        issue_stage(a, stage_info(a, u0, u1, tile_units, i + a.depth), swiglu, lane,
                    stages + slot * kTileRows * row_bytes, &bars[slot]);
      // The ordered chain: one lane per physical row, groups ascending.
#pragma unroll
      for (int g = 0; g < kMaxGroupsPerChunk; g++)
        if (g < groups)
          acc = __fmaf_rn(Tb[g * kTileRows + lane], wcur[g], acc);
      if (s.chunk == a.nchunks - 1) {
        float gate = __shfl_down_sync(0xffffffffu, acc, 16);
        if (swiglu) {
          if (lane < s.cnt) {
            RowRef r = row_of(a, s.ub + lane, false);
            r.out[r.local] = silu_gate_dev(acc, gate);
          }
        } else if (lane < s.cnt) {
          RowRef r = row_of(a, s.ub + lane, false);
          if (a.kind == KC_ADD)
            r.out[r.local] = __fadd_rn(r.out[r.local], acc);
          else
            r.out[r.local] = acc;
        }
        acc = 0.0f;
      }
#pragma unroll
      for (int g = 0; g < kMaxGroupsPerChunk; g++)
        wcur[g] = wnext[g];
    }
  }
  // After an abort, let the copies this CTA issued (stages aborted_at .. aborted_at + depth - 1) land, with bounded
  // waits, before its shared memory goes away.
  if (aborted_at >= 0 && tid == 0)
    for (int j = aborted_at; j < S && j < aborted_at + a.depth; j++)
      mbar_wait_bounded(&bars[j % a.depth], (unsigned)(j / a.depth) & 1u);
}

}  // namespace

size_t kc_gemv_smem_bytes(int n, int gs, int kc, int depth) {
  return 256 + (size_t)((n / gs * 4 + 15) & ~15) + (size_t)((n + 15) & ~15) +
         (size_t)2 * kMaxGroupsPerChunk * kTileRows * 4 + (size_t)depth * kTileRows * (kc + kPad);
}

// Host launcher (argument validation is the C-ABI layer's job).
int kc_launch_gemv(const KcGemvSeg *segs, int nseg, const int8_t *xq, const float *xs, int n, long long ld, int gs,
                   int kind, cudaStream_t stream, int grid_limit) {
  GemvArgs a = {};
  int units = 0;
  bool vec4 = ((ld / gs) % 4) == 0;
  for (int s = 0; s < nseg; s++) {
    a.seg[s].out = segs[s].out;
    a.seg[s].wq = segs[s].wq;
    a.seg[s].ws = segs[s].ws;
    a.seg[s].w3q = segs[s].w3q;
    a.seg[s].w3s = segs[s].w3s;
    a.seg[s].d = segs[s].d;
    a.seg[s].unit0 = units;
    units += segs[s].d;
    vec4 = vec4 && ((uintptr_t)segs[s].ws % 16 == 0) && (!segs[s].w3s || (uintptr_t)segs[s].w3s % 16 == 0);
  }
  if (units == 0 || n == 0)
    return 0;
  a.nseg = nseg;
  a.xq = xq;
  a.xs = xs;
  a.n = n;
  a.ld = ld;
  a.gs = gs;
  a.kind = kind;
  a.units = units;
  a.kc = gs >= 32 ? 1024 : 512;
  if (a.kc < gs)
    a.kc = gs;
  a.nchunks = (n + a.kc - 1) / a.kc;
  a.ws_vec4 = vec4 ? 1 : 0;
  const size_t budget = 220 * 1024;
  size_t fixed = kc_gemv_smem_bytes(n, gs, a.kc, 0);
  size_t per_stage = (size_t)kTileRows * (a.kc + kPad);
  if (fixed + 2 * per_stage > budget)
    return -1;
  int depth = (int)((budget - fixed) / per_stage);
  a.depth = depth > 6 ? 6 : depth;
  size_t smem = kc_gemv_smem_bytes(n, gs, a.kc, a.depth);
  int sms = kc_device_sms();
  int grid = units < sms ? units : sms;
  if (grid_limit > 0 && grid > grid_limit)
    grid = grid_limit;
  static bool attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(gemv_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr_set[dev] = true;
  }
  gemv_q8_kernel<<<grid, kThreads, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
