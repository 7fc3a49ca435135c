// Q8_0 W8A8 prefill GEMM for sm_100a on the 5th-generation tensor core:
//   C[m][n] (op)= sum over 64-groups g of (float)dot_g(xq[m], wq[n]) * xs[m][g] * ws[n][g]
// with the epilogues of the reference's batched GEMM (q8_gemm_chunks, src/gemm.c:963-989: STORE / ADD / PARTIAL, and
// SWIGLU on a w1/w3 pair) over 1-3 segments that share the activations (k_gemm_q8, include/gemm.h:130-133).
//
// Arithmetic, bitwise the reference's AMX-INT8 backend (amx_q8_chunk, src/gemm.c:564-608) and this library's GEMV:
// every group dot is an exact int32 (tcgen05.mma kind::i8, two K=32 steps per 64-group), and every output rescales
// the groups in ascending order as acc = fmaf((float)dot * xs, ws, acc) from acc = 0.
//
// Tiling: the MMA's M side is 128 weight rows (64 w1 + 64 w3 rows for SwiGLU), its N side 128 tokens; a persistent
// CTA per SM walks its tiles (tokens fastest, so the CTAs running together share weight stripes in L2).
//   warp 0      TMA producer: per stage (two groups, 128 B of K) one [128 x 128 B] weight box, one [128 x 128 B]
//               activation box (both 128B-swizzled, the canonical K-major UMMA layout) and the stage's transposed
//               activation scales [2 groups x 128 tokens]; a ring of 4 stages.
//   warp 1      MMA issuer: allocates 256 TMEM columns (two 128 x 128 int32 buffers), issues two MMAs per group into
//               the buffer the epilogue has released, commits the buffer to the epilogue and the stage to the ring.
//   warps 4-11  epilogue (warp % 4 = TMEM lane quadrant = 32 weight rows, (warp - 4) / 4 = 64-token half): per
//               group it reads its 32 x 64 int32 dots and promotes them with packed f32x2 instructions, then refills
//               its part of the buffer with the exponent bias and releases it.
// Group promotion without integer->float conversions: each buffer holds the int32 pattern of 1.5 * 2^23 before the
// group's MMAs accumulate onto it, so the result read back IS the float 1.5 * 2^23 + dot exactly (|dot| <= 64*127^2
// < 2^22); one subtraction recovers (float)dot. The promotion is then sub, mul, fma per pair of outputs.
//
// Every mbarrier wait is bounded (a timeout raises KC_ERR_TIMEOUT, sets a CTA abort flag that turns the remaining
// waits into no-ops, and the CTA still releases its TMEM).
#include <cuda.h>
#include <string.h>

#include "common.cuh"
#include "kernels_cuda_internal.h"
#include "tcgen05.cuh"
#include "tmap.h"

namespace {

constexpr int kTM = 128;                      // weight rows per tile (MMA M)
constexpr int kTN = 128;                      // tokens per tile (MMA N)
constexpr int kStages = 4;
constexpr int kStageA = kTM * 128;            // weights: 128 rows x 128 B
constexpr int kStageB = kTN * 128;            // activations: 128 tokens x 128 B
constexpr int kStageX = 2 * kTN * 4;          // activation scales: 2 groups x 128 tokens
constexpr int kStageBytes = kStageA + kStageB + 1024;
constexpr int kXchBytes = kTN * 64 * 4;       // SwiGLU exchange: 128 tokens x 64 w3 rows
constexpr int kThreads = 12 * 32;
constexpr int kEpiWarp0 = 4;
constexpr int kEpiWarps = 8;
constexpr int kTmemCols = 256;
constexpr uint32_t kBiasBits = 0x4B400000u;   // 1.5 * 2^23
constexpr float kBias = 12582912.0f;
constexpr int kBarXchFull = 1, kBarXchFree = 2;  // named barriers among the epilogue warps

struct __align__(64) GemmMaps {
  CUtensorMap w[3];  // weights per segment (w1 for SwiGLU): boxes [128 B x 128 rows] (64 rows for SwiGLU)
  CUtensorMap w3;    // SwiGLU second matrix
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
  if (mbar_wait_bounded(bar, parity))
    return true;
  *abort_flag = 1;
  return false;
}

__device__ __forceinline__ void bar_sync_epi(int id) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(kEpiWarps * 32) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) gemm_q8_tc_kernel(const __grid_constant__ GemmMaps mp, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  // The 128-byte swizzle is a function of the address bits, so the operand stages start on a 1024-byte boundary.
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t *stages = smem;
  float *xch = reinterpret_cast<float *>(smem + kStages * kStageBytes);
  uint8_t *tail = smem + kStages * kStageBytes + kXchBytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(tail);
  uint64_t *empty = full + kStages;
  uint64_t *tfull = empty + kStages;
  uint64_t *tempty = tfull + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
  volatile int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1 + kEpiWarps);
    }
    for (int i = 0; i < 2; i++) {
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

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    int st = 0;
    for (int t = blockIdx.x; t < a.total_tiles; t += G) {
      const Tile tl = decode_tile(a, t);
      for (int j = 0; j < spt; j++, st++) {
        const int slot = st % kStages, use = st / kStages;
        if (!wait_or_abort(&empty[slot], (use & 1) ^ 1, abort_flag))
          continue;
        uint8_t *base = stages + slot * kStageBytes;
        mbar_arrive_expect_tx(&full[slot], kStageA + kStageB + kStageX);
        const int k0 = j * 128;
        if (tl.swiglu) {
          tma_load_2d(base, &mp.w[0], k0, tl.n0, &full[slot]);
          tma_load_2d(base + kStageA / 2, &mp.w3, k0, tl.n0, &full[slot]);
        } else {
          tma_load_2d(base, &mp.w[0] + tl.s, k0, tl.n0, &full[slot]);
        }
        tma_load_2d(base + kStageA, &mp.x, k0, tl.m0, &full[slot]);
        tma_load_2d(base + kStageA + kStageB, &mp.xs, tl.m0, 2 * j, &full[slot]);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
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
          const int b = gidx & 1, ub = gidx >> 1;
          const bool ok = wait_or_abort(&tempty[b], ub & 1, abort_flag) && have;
          tc_fence_after();
          if (ok) {
#pragma unroll
            for (int k = 0; k < 2; k++) {
              const uint64_t off = (uint64_t)((gg * 64 + k * 32) >> 4);
              umma_i8(tmem + b * kTN, adesc + off, bdesc + off, idesc, true);
            }
          }
          umma_commit(&tfull[b]);
        }
        umma_commit(&empty[slot]);
      }
    }
  } else if (warp >= kEpiWarp0) {
    // ---- epilogue: promotion of every group, in order ----
    const int q = warp & 3, h = (warp - kEpiWarp0) >> 2;
    const int row = 32 * q + lane;  // TMEM lane = row of the weight tile
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + 64 * h;
    // Both buffers start out holding the bias.
    tmem_st32_fill(tq, kBiasBits);
    tmem_st32_fill(tq + 32, kBiasBits);
    tmem_st32_fill(tq + kTN, kBiasBits);
    tmem_st32_fill(tq + kTN + 32, kBiasBits);
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&tempty[0]);
      mbar_arrive(&tempty[1]);
    }
    const uint64_t negbias2 = f2_pack(-kBias, -kBias);
    int st = 0, gidx = 0;
    for (int t = blockIdx.x; t < a.total_tiles; t += G) {
      const Tile tl = decode_tile(a, t);
      const GemmSegDev sg = tl.s == 0 ? a.seg[0] : tl.s == 1 ? a.seg[1] : a.seg[2];
      const bool w3row = tl.swiglu && row >= kTM / 2;
      const int n = tl.n0 + (tl.swiglu ? (row & (kTM / 2 - 1)) : row);
      const bool row_ok = n < sg.n;
      const float *wsr = (w3row ? sg.ws3 : sg.ws) + (size_t)min(n, sg.n - 1) * groups;
      float4 w_cur = __ldg(reinterpret_cast<const float4 *>(wsr));
      float4 w_n1 = groups > 4 ? __ldg(reinterpret_cast<const float4 *>(wsr + 4)) : w_cur;
      float4 w_n2 = groups > 8 ? __ldg(reinterpret_cast<const float4 *>(wsr + 8)) : w_cur;
      uint64_t acc[32];
#pragma unroll
      for (int i = 0; i < 32; i++)
        acc[i] = 0;
      for (int j = 0; j < spt; j++, st++) {
        const int slot = st % kStages, use = st / kStages;
        wait_or_abort(&full[slot], use & 1, abort_flag);
        const float *xsT = reinterpret_cast<const float *>(stages + slot * kStageBytes + kStageA + kStageB);
        for (int gg = 0; gg < 2 && 2 * j + gg < groups; gg++, gidx++) {
          const int g = 2 * j + gg;
          const int b = gidx & 1, ub = gidx >> 1;
          const bool ok = wait_or_abort(&tfull[b], ub & 1, abort_flag);
          tc_fence_after();
          if ((g & 3) == 0 && g > 0) {
            w_cur = w_n1;
            w_n1 = w_n2;
            if (g + 8 < groups)
              w_n2 = __ldg(reinterpret_cast<const float4 *>(wsr + g + 8));
          }
          const float wv = (g & 3) == 0 ? w_cur.x : (g & 3) == 1 ? w_cur.y : (g & 3) == 2 ? w_cur.z : w_cur.w;
          const uint64_t ws2 = f2_pack(wv, wv);
          const float4 *xs4 = reinterpret_cast<const float4 *>(xsT + gg * kTN + 64 * h);
          // Two halves of 32 columns: read, promote, then refill the buffer with the bias and release it.
#pragma unroll
          for (int half = 0; half < 2; half++) {
            uint32_t r[32];
            tmem_ld32(tq + b * kTN + 32 * half, r);
            tmem_wait_ld();
            if (!ok)
              continue;
            if (a.dots) {
              if (row_ok && tl.s == 0 && !tl.swiglu)
                for (int c = 0; c < 32; c++) {
                  const int m = tl.m0 + 64 * h + 32 * half + c;
                  if (m < a.M)
                    a.dots[((size_t)g * a.M + m) * sg.n + n] = (int32_t)(r[c] - kBiasBits);
                }
              continue;
            }
#pragma unroll
            for (int c4 = 0; c4 < 8; c4++) {
              const float4 x = xs4[8 * half + c4];
              const int c = 4 * c4;
              uint64_t f0 = f2_add(f2_pack_bits(r[c], r[c + 1]), negbias2);
              uint64_t f1 = f2_add(f2_pack_bits(r[c + 2], r[c + 3]), negbias2);
              f0 = f2_mul(f0, f2_pack(x.x, x.y));
              f1 = f2_mul(f1, f2_pack(x.z, x.w));
              acc[16 * half + 2 * c4] = f2_fma(f0, ws2, acc[16 * half + 2 * c4]);
              acc[16 * half + 2 * c4 + 1] = f2_fma(f1, ws2, acc[16 * half + 2 * c4 + 1]);
            }
          }
          tmem_st32_fill(tq + b * kTN, kBiasBits);
          tmem_st32_fill(tq + b * kTN + 32, kBiasBits);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0)
            mbar_arrive(&tempty[b]);
        }
        __syncwarp();
        if (lane == 0)
          mbar_arrive(&empty[slot]);
      }
      if (a.dots)
        continue;
      // ---- write the tile: thread = weight row n, 64 tokens ----
      const int mbase = tl.m0 + 64 * h;
      if (tl.swiglu) {
        if (w3row) {
#pragma unroll
          for (int i = 0; i < 32; i++) {
            float lo, hi;
            f2_unpack(acc[i], lo, hi);
            xch[(64 * h + 2 * i) * 64 + (row - kTM / 2)] = lo;
            xch[(64 * h + 2 * i + 1) * 64 + (row - kTM / 2)] = hi;
          }
        }
        bar_sync_epi(kBarXchFull);
        if (!w3row && row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i++) {
            float lo, hi;
            f2_unpack(acc[i], lo, hi);
            const int m = mbase + 2 * i;
            if (m < a.M)
              sg.c[(size_t)m * sg.ldc + n] = silu_gate_dev(lo, xch[(64 * h + 2 * i) * 64 + row]);
            if (m + 1 < a.M)
              sg.c[(size_t)(m + 1) * sg.ldc + n] = silu_gate_dev(hi, xch[(64 * h + 2 * i + 1) * 64 + row]);
          }
        }
        bar_sync_epi(kBarXchFree);
      } else if (row_ok) {
#pragma unroll
        for (int i = 0; i < 32; i++) {
          float lo, hi;
          f2_unpack(acc[i], lo, hi);
          const int m = mbase + 2 * i;
          float *c0 = sg.c + (size_t)m * sg.ldc + n;
          if (m < a.M)
            *c0 = sg.kind == KC_ADD ? __fadd_rn(*c0, lo) : lo;
          if (m + 1 < a.M)
            c0[sg.ldc] = sg.kind == KC_ADD ? __fadd_rn(c0[sg.ldc], hi) : hi;
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
  transpose_scales_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(xsT, xs, M, groups, ldt);
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
      if (!kc_tmap_2d(&mp.w[0], segs[s].wq, 1, K, segs[s].n, K, 128, kTM / 2, true) ||
          !kc_tmap_2d(&mp.w3, segs[s].w3q, 1, K, segs[s].n, K, 128, kTM / 2, true))
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
  const size_t smem = (size_t)kStages * kStageBytes + kXchBytes + 256 + 1024;
  static bool attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(gemm_q8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr_set[dev] = true;
  }
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
  return cudaLaunchKernelEx(&cfg, gemm_q8_tc_kernel, mp, a) == cudaSuccess ? 0 : -2;
}
