// Activation quantizer, RMSNorm (+ fused quantize) and RoPE for sm_100a.
//
// - quantize_rows_kernel: k_quantize / k_quantize_rows (src/gemv.c:589-624, src/gemm.c:818-830), one warp per group.
//   max|x| is exact in any order; the scale is the IEEE quotient max / 127.0f and each value is
//   roundf(clamp(x / scale)), so the int8 values and scales are bitwise the reference's on every ISA.
// - rmsnorm_kernel: rmsnorm_avx512's order (src/kernels_simd.c:136-161), reproduced lane for lane: 64 threads keep
//   the four 16-lane FMA accumulators over 64-value steps (tail into the first), then (a0+a1)+(a2+a3) and GCC's
//   _mm512_reduce_add_ps tree, then ss / size + eps, 1 / sqrtf, o = w * (ss * x). With `q` set, the output is also
//   quantized in gs-groups in the same kernel (the k_rmsnorm -> k_quantize pair of src/tp.c:403-404 fused).
// - rope_rows_kernel: k_rope_apply (src/kernels_simd.c:203-227): a*c - b*s and a*s + b*c without contraction, from a
//   host-computed table (k_rope_table), so the rotation is bitwise the reference's.
#include "common.cuh"
#include "kernels_cuda_internal.h"

namespace {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__global__ void quantize_rows_kernel(int8_t *q, float *s, const float *x, long long ldx, int m, int n, int gs) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = n / gs;
  const long long gid = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
  if (gid >= (long long)m * groups)
    return;
  const int row = (int)(gid / groups), g = (int)(gid - (long long)row * groups);
  const float *xg = x + row * ldx + (long long)g * gs;
  float mx = 0.0f;
  int bad = 0;
  for (int i = lane; i < gs; i += 32) {
    float v = xg[i];
    bad |= !isfinite(v);
    mx = fmaxf(mx, fabsf(v));
  }
  if (__any_sync(0xffffffffu, bad)) {
    if (lane == 0)
      kc_raise(KC_ERR_NONFINITE);
    return;
  }
  mx = warp_max(mx);
  const float scale = __fdiv_rn(mx, 127.0f);
  if (lane == 0)
    s[(long long)row * groups + g] = scale;
  int8_t *qg = q + (long long)row * n + (long long)g * gs;
  for (int i = lane; i < gs; i += 32)
    qg[i] = (int8_t)quantize_value(xg[i], scale);
}

// gs = 64 (the checkpoints' group size): a warp quantizes kQuantGroupsPerWarp groups, each lane a float2 of every
// group, all loads in flight before the first reduction; per element the arithmetic is quantize_rows_kernel's.
constexpr int kQuantGroupsPerWarp = 4;

__global__ void quantize_rows64_kernel(int8_t *q, float *s, const float *x, long long ldx, int m, int n) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = n / 64;
  const long long total = (long long)m * groups;
  const long long g0 = ((long long)blockIdx.x * (blockDim.x >> 5) + warp) * kQuantGroupsPerWarp;
  float2 v[kQuantGroupsPerWarp];
#pragma unroll
  for (int k = 0; k < kQuantGroupsPerWarp; k++) {
    const long long gid = g0 + k;
    if (gid < total) {
      const long long row = gid / groups, g = gid - row * groups;
      v[k] = *reinterpret_cast<const float2 *>(x + row * ldx + g * 64 + 2 * lane);
    }
  }
#pragma unroll
  for (int k = 0; k < kQuantGroupsPerWarp; k++) {
    const long long gid = g0 + k;
    if (gid >= total)
      break;
    const long long row = gid / groups, g = gid - row * groups;
    const int bad = !isfinite(v[k].x) || !isfinite(v[k].y);
    if (__any_sync(0xffffffffu, bad)) {
      if (lane == 0)
        kc_raise(KC_ERR_NONFINITE);
      continue;
    }
    const float mx = warp_max(fmaxf(fabsf(v[k].x), fabsf(v[k].y)));
    const float scale = __fdiv_rn(mx, 127.0f);
    if (lane == 0)
      s[row * groups + g] = scale;
    char2 c;
    c.x = (signed char)quantize_value(v[k].x, scale);
    c.y = (signed char)quantize_value(v[k].y, scale);
    *reinterpret_cast<char2 *>(q + row * n + g * 64 + 2 * lane) = c;
  }
}

// gs = 64 with 16-byte rows: a half-warp per group, each lane a float4 of it, a warp taking kQuant4Groups groups with
// every load in flight before the first reduction (the group maximum is four shuffles within the half-warp); per
// element the arithmetic is quantize_rows_kernel's.
constexpr int kQuant4Groups = 8;

__global__ void quantize_rows64x4_kernel(int8_t *q, float *s, const float *x, long long ldx, int m, int n) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, half = lane >> 4, l16 = lane & 15;
  const int groups = n / 64;
  const long long total = (long long)m * groups;
  const long long g0 = ((long long)blockIdx.x * (blockDim.x >> 5) + warp) * kQuant4Groups;
  float4 v[kQuant4Groups / 2];
#pragma unroll
  for (int k = 0; k < kQuant4Groups / 2; k++) {
    const long long gid = g0 + 2 * k + half;
    if (gid < total) {
      const long long row = gid / groups, g = gid - row * groups;
      v[k] = *reinterpret_cast<const float4 *>(x + row * ldx + g * 64 + 4 * l16);
    }
  }
#pragma unroll
  for (int k = 0; k < kQuant4Groups / 2; k++) {
    const long long gid = g0 + 2 * k + half;
    const bool live = gid < total;
    const int bad = live && (!isfinite(v[k].x) || !isfinite(v[k].y) || !isfinite(v[k].z) || !isfinite(v[k].w));
    const unsigned ballot = __ballot_sync(0xffffffffu, bad);
    float mx = live ? fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))) : 0.0f;
#pragma unroll
    for (int o = 8; o; o >>= 1)
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (!live)
      continue;
    if ((ballot >> (16 * half)) & 0xFFFFu) {
      if (l16 == 0)
        kc_raise(KC_ERR_NONFINITE);
      continue;
    }
    const long long row = gid / groups, g = gid - row * groups;
    const float scale = __fdiv_rn(mx, 127.0f);
    if (l16 == 0)
      s[row * groups + g] = scale;
    char4 c;
    c.x = (signed char)quantize_value(v[k].x, scale);
    c.y = (signed char)quantize_value(v[k].y, scale);
    c.z = (signed char)quantize_value(v[k].z, scale);
    c.w = (signed char)quantize_value(v[k].w, scale);
    *reinterpret_cast<char4 *>(q + row * n + g * 64 + 4 * l16) = c;
  }
}

constexpr int kNormThreads = 256;
constexpr int kMaxValuesPerLane = 8;    // fused quantize: gs <= 256
constexpr int kNormStagedMax = 16384;   // sizes whose row is staged in shared memory (64 KB)

// Copies n floats (global, any alignment) to shared memory with all threads, each keeping 8 loads in flight before
// its first store (a load-then-store loop would wait one memory round trip per element).
__device__ __forceinline__ void stage_row(float *dst, const float *src, int n) {
  constexpr int B = 8;
  if ((((uintptr_t)src) & 15) == 0 && (n & 3) == 0) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 *d4 = reinterpret_cast<float4 *>(dst);
    for (int base = threadIdx.x; base < n / 4; base += kNormThreads * B) {
      float4 r[B];
#pragma unroll
      for (int b = 0; b < B; b++)
        if (base + b * kNormThreads < n / 4)
          r[b] = s4[base + b * kNormThreads];
#pragma unroll
      for (int b = 0; b < B; b++)
        if (base + b * kNormThreads < n / 4)
          d4[base + b * kNormThreads] = r[b];
    }
  } else {
    for (int base = threadIdx.x; base < n; base += kNormThreads * B) {
      float r[B];
#pragma unroll
      for (int b = 0; b < B; b++)
        if (base + b * kNormThreads < n)
          r[b] = src[base + b * kNormThreads];
#pragma unroll
      for (int b = 0; b < B; b++)
        if (base + b * kNormThreads < n)
          dst[base + b * kNormThreads] = r[b];
    }
  }
}

// One CTA per row. With STAGED the row and the weights are first copied to shared memory (2 * size floats of dynamic
// shared memory); without, they are read from global memory (sizes beyond kNormStagedMax).
template <bool STAGED>
__global__ void __launch_bounds__(kNormThreads, 5) rmsnorm_kernel(float *out, int8_t *q, float *s, const float *x,
                                                                const float *w, int size, long long ldx, float eps,
                                                                int gs) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) float norm_dyn[];
  __shared__ float lanes[64];
  __shared__ float inv;
  const int tid = threadIdx.x, row = blockIdx.x;
  const float *xr = x + row * ldx;
  if (STAGED) {  // the row only: the weights are the same for every row, so every CTA of the SM reads them cached
    stage_row(norm_dyn, xr, size);
    __syncthreads();
    xr = norm_dyn;
  }
  if (tid < 64)
    lanes[tid] = rms_lane_sum(xr, size, tid);
  __syncthreads();
  if (tid == 0)
    inv = rms_inverse(lanes, size, eps);
  __syncthreads();
  const float ss = inv;
  if (!q) {
    float *orow = out + (long long)row * size;
    for (int j = tid; j < size; j += kNormThreads)
      orow[j] = rms_apply(xr[j], w[j], ss);
    return;
  }
  const int warp = tid >> 5, lane = tid & 31, groups = size / gs;
  for (int g = warp; g < groups; g += kNormThreads / 32) {
    float o[kMaxValuesPerLane];
    float mx = 0.0f;
#pragma unroll
    for (int t = 0; t < kMaxValuesPerLane; t++) {
      int i = lane + 32 * t;
      if (i < gs) {
        int j = g * gs + i;
        o[t] = rms_apply(xr[j], w[j], ss);
        mx = fmaxf(mx, fabsf(o[t]));
      }
    }
    int bad = 0;
#pragma unroll
    for (int t = 0; t < kMaxValuesPerLane; t++)
      if (lane + 32 * t < gs)
        bad |= !isfinite(o[t]);
    if (__any_sync(0xffffffffu, bad)) {
      if (lane == 0)
        kc_raise(KC_ERR_NONFINITE);
      return;
    }
    mx = warp_max(mx);
    const float scale = __fdiv_rn(mx, 127.0f);
    if (lane == 0)
      s[(long long)row * groups + g] = scale;
#pragma unroll
    for (int t = 0; t < kMaxValuesPerLane; t++) {
      int i = lane + 32 * t;
      if (i < gs) {
        long long j = (long long)g * gs + i;
        q[(long long)row * size + j] = (int8_t)quantize_value(o[t], scale);
        if (out)
          out[(long long)row * size + j] = o[t];
      }
    }
  }
}

__global__ void rope_rows_kernel(float *q, long long q_stride, float *k, long long k_stride, const float *table,
                                 long long table_stride, int rows, int n_heads, int n_kv_heads, int head_dim) {
  pdl_wait();
  pdl_launch_dependents();
  const int half = head_dim / 2;
  const int per_row = (n_heads + n_kv_heads) * half;
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (long long)rows * per_row)
    return;
  const int row = (int)(id / per_row);
  int p = (int)(id - (long long)row * per_row);
  float *v;
  if (p < n_heads * half) {
    v = q + row * q_stride;
  } else {
    p -= n_heads * half;
    v = k + row * k_stride;
  }
  const int h = p / half, j = 2 * (p - h * half);
  const float *t = table + row * table_stride;
  const float c = t[j], sn = t[head_dim + j + 1];
  float *e = v + (long long)h * head_dim + j;
  const float a = e[0], b = e[1];
  e[0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
  e[1] = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
}

}  // namespace

int kc_launch_quantize_rows(int8_t *q, float *s, const float *x, long long ldx, int m, int n, int gs,
                            cudaStream_t stream) {
  long long groups = (long long)m * (n / gs);
  if (groups == 0)
    return 0;
  const int warps = 8;
  if (gs == 64 && ((uintptr_t)x & 15) == 0 && (ldx & 3) == 0 && ((uintptr_t)q & 3) == 0 && (n & 3) == 0) {
    const long long per_block = (long long)warps * kQuant4Groups;
    kc_launch_pdl(quantize_rows64x4_kernel, (unsigned)((groups + per_block - 1) / per_block), warps * 32, 0, stream,
                  q, s, x, ldx, m, n);
  } else if (gs == 64 && ((uintptr_t)x & 7) == 0 && (ldx & 1) == 0 && ((uintptr_t)q & 1) == 0) {
    const long long per_block = (long long)warps * kQuantGroupsPerWarp;
    kc_launch_pdl(quantize_rows64_kernel, (unsigned)((groups + per_block - 1) / per_block), warps * 32, 0, stream, q,
                  s, x, ldx, m, n);
  } else {
    kc_launch_pdl(quantize_rows_kernel, (unsigned)((groups + warps - 1) / warps), warps * 32, 0, stream, q, s, x, ldx,
                  m, n, gs);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int kc_launch_rmsnorm(float *out, int8_t *q, float *s, const float *x, const float *w, int rows, int size,
                      long long ldx, float eps, int gs, cudaStream_t stream) {
  if (rows == 0 || size == 0)
    return 0;
  if (q && (gs <= 0 || gs > 32 * kMaxValuesPerLane || size % gs))
    return -1;
  if (size <= kNormStagedMax) {
    const int bytes = size * (int)sizeof(float);
    // Raised once per device to the largest staged row (kc_allow_smem keeps its own locked record).
    if (bytes > 48 * 1024 && kc_allow_smem(reinterpret_cast<const void *>(rmsnorm_kernel<true>),
                                           kNormStagedMax * (int)sizeof(float)) != cudaSuccess)
      return -2;
    kc_launch_pdl(rmsnorm_kernel<true>, rows, kNormThreads, bytes, stream, out, q, s, x, w, size, ldx, eps, gs);
  } else {
    kc_launch_pdl(rmsnorm_kernel<false>, rows, kNormThreads, 0, stream, out, q, s, x, w, size, ldx, eps, gs);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int kc_launch_rope_rows(float *q, long long q_stride, float *k, long long k_stride, const float *table,
                        long long table_stride, int rows, int n_heads, int n_kv_heads, int head_dim,
                        cudaStream_t stream) {
  long long total = (long long)rows * (n_heads + n_kv_heads) * (head_dim / 2);
  if (total == 0)
    return 0;
  kc_launch_pdl(rope_rows_kernel, (unsigned)((total + 255) / 256), 256, 0, stream, q, q_stride, k, k_stride, table,
                                                                          table_stride, rows, n_heads, n_kv_heads,
                                                                          head_dim);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
