// Shared device helpers for the sm_100a Q8_0 kernels: the device error word, bounded mbarrier waits, 1-D bulk
// (TMA) copies, and the exact float epilogues the reference's C source implies.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

// Error bits the kernels set in the per-device error word (read back by the C-ABI layer, kc_status()).
enum : unsigned {
  KC_ERR_NONFINITE = 1u,   // k_quantize met a non-finite activation (src/gemv.c:599-600 fails the same way)
  KC_ERR_TIMEOUT = 2u,     // a bounded wait on an mbarrier or flag gave up
  KC_ERR_BAD_ARGS = 4u,    // a kernel was launched with arguments its host checks should have refused
};

// One word per device, in the library's own device memory; kernels OR error bits into it.
extern __device__ unsigned kc_error_word;

__device__ __forceinline__ void kc_raise(unsigned bits) { atomicOr(&kc_error_word, bits); }

__device__ __forceinline__ uint64_t kc_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Every spin in this library gives up after this many nanoseconds and raises KC_ERR_TIMEOUT.
constexpr uint64_t KC_WAIT_NS = 2000000000ull;

// Slots of the peer reductions: 8-byte {float bits, call number} words written and polled whole, in this GPU's memory
// or a peer's (CUDA IPC mapping); volatile, so every poll reads memory.
__device__ __forceinline__ unsigned long long peer_ld_slot(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void peer_st_slot(unsigned long long *p, unsigned long long v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete; false (and KC_ERR_TIMEOUT raised) after KC_WAIT_NS.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, unsigned parity) {
  if (mbar_try_wait(bar, parity))
    return true;
  uint64_t start = kc_globaltimer();
  for (unsigned i = 1;; i++) {
    if (mbar_try_wait(bar, parity))
      return true;
    if ((i & 255u) == 0 && kc_globaltimer() - start > KC_WAIT_NS) {
      kc_raise(KC_ERR_TIMEOUT);
      return false;
    }
  }
}

// The same wait for threads that share an SM sub-partition with busy warps: each try_wait suspends the thread in
// hardware (up to `hint_ns`, waking when the phase completes) instead of spinning on the issue port.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, unsigned parity, unsigned hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_sleep_bounded(uint64_t *bar, unsigned parity) {
  if (mbar_try_wait_sleep(bar, parity, 1000u))
    return true;
  uint64_t start = kc_globaltimer();
  for (unsigned i = 1;; i++) {
    if (mbar_try_wait_sleep(bar, parity, 1000u))
      return true;
    if ((i & 15u) == 0 && kc_globaltimer() - start > KC_WAIT_NS) {
      kc_raise(KC_ERR_TIMEOUT);
      return false;
    }
  }
}

// 1-D bulk copy global -> shared through the TMA unit, completing `bytes` of transaction count on `bar`.
// dst and src 16-byte aligned, bytes a multiple of 16; the destination is this CTA's shared memory only.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled TMA load of the box at (x, y) (x in elements of the innermost dimension; x * element size must be a
// multiple of 16 bytes) into shared memory, completing its bytes on `bar` (this CTA only).
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled TMA load of the box at (x, y, z) into shared memory, completing its bytes on `bar` (this CTA only).
__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap, int x, int y, int z, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its independent prologue now, and wait for
// the previous kernel's results. Both are no-ops unless the launch carries the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ int4 lds128(const void *p) {
  int4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ int dot16(int4 a, int4 b, int acc) {
  acc = __dp4a(a.x, b.x, acc);
  acc = __dp4a(a.y, b.y, acc);
  acc = __dp4a(a.z, b.z, acc);
  acc = __dp4a(a.w, b.w, acc);
  return acc;
}

// expf as the reference's C library computes it: glibc's expf (2.28 and later, this image's 2.39: the published method
// of its sysdeps/ieee754/flt-32/e_expf.c, from Arm's optimized-routines). In double precision: z = x * 32 / ln 2,
// k = z rounded to an integer by adding and subtracting 1.5 * 2^52, r = z - k, 2^(k/32) from a table of 2^(i/32)
// (T[i] = bits(2^(i/32)) - (i << 47), every entry the correctly rounded double) with k >> 5 added to the exponent,
// times the cubic C0 r^3 + C1 r^2 + C2 r + 1 evaluated as written (no fused multiply-add: glibc's generic x86-64
// build), rounded once to float. Below log(2^-150) the result is 0, above log(2^128) infinity, as glibc returns.
// Bitwise glibc's expf on every input checked (3 million, the softmax and SiLU ranges); a correctly rounded exp
// differs from it on about 1 input in 1600, which is why the table method is restated rather than exp(double) used.
static __constant__ unsigned long long kExpfTable[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

__device__ __forceinline__ float expf_libc(float x) {
  if (x < -0x1.9fe368p6f)
    return 0.0f;
  if (x > 0x1.62e42ep6f)
    return __int_as_float(0x7f800000);
  const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32,
               c2 = 0x1.62e42ff0c52d6p-1 / 32, inv_ln2_n = 0x1.71547652b82fep+0 * 32, shift = 0x1.8p+52;
  const double z = __dmul_rn(inv_ln2_n, (double)x);
  double kd = __dadd_rn(z, shift);
  const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
  kd = __dsub_rn(kd, shift);
  const double r = __dsub_rn(z, kd);
  const double s = __longlong_as_double((long long)(kExpfTable[ki % 32] + (ki << 47)));
  const double zz = __dadd_rn(__dmul_rn(c0, r), c1), r2 = __dmul_rn(r, r);
  double y = __dadd_rn(__dmul_rn(c2, r), 1.0);
  y = __dadd_rn(__dmul_rn(zz, r2), y);
  return __double2float_rn(__dmul_rn(y, s));
}

// silu_gate (src/gemv.c:246-250): value *= 1 / (1 + expf(-value)); value * gate, with the C library's expf.
__device__ __forceinline__ float silu_gate_dev(float value, float gate) {
  const float e = expf_libc(-value);
  value = __fmul_rn(value, __fdiv_rn(1.0f, __fadd_rn(1.0f, e)));
  return __fmul_rn(value, gate);
}

// RMSNorm's sum of squares in the reference's AVX-512 order (src/kernels_simd.c:136-161): 64 lanes, lane l
// accumulating x[l], x[64 + l], ... with FMAs, a 16-lane tail for sizes that are not a multiple of 64. Call from
// threads 0..63; returns lane l's partial. Unrolled 16 deep so a lane's loads run ahead of its FMA chain (the fused
// GEMV prologue waits on this: decode step 2.379 ms at 8, 2.365 ms at 16, 2.420 ms at 2).
__device__ __forceinline__ float rms_lane_sum(const float *x, int size, int l) {
  float a = 0.0f;
  int j = 0;
#pragma unroll 16
  for (; j + 64 <= size; j += 64)
    a = __fmaf_rn(x[j + l], x[j + l], a);
  if (l < 16)
    for (; j < size; j += 16)
      if (j + l < size)
        a = __fmaf_rn(x[j + l], x[j + l], a);
  return a;
}

// The 64 lane partials reduced in the reference's order ((a0 + a1) + (a2 + a3) per 16-lane group, then GCC's
// reduce_add_ps tree), divided by size, plus epsilon: 1 / sqrtf of that (one thread).
__device__ __forceinline__ float rms_inverse(const float *lanes, int size, float eps) {
  float v[16], t8[8], t4[4];
  for (int l = 0; l < 16; l++)
    v[l] = __fadd_rn(__fadd_rn(lanes[l], lanes[16 + l]), __fadd_rn(lanes[32 + l], lanes[48 + l]));
  for (int l = 0; l < 8; l++)
    t8[l] = __fadd_rn(v[8 + l], v[l]);
  for (int l = 0; l < 4; l++)
    t4[l] = __fadd_rn(t8[4 + l], t8[l]);
  float ss = __fadd_rn(__fadd_rn(t4[0], t4[2]), __fadd_rn(t4[1], t4[3]));
  ss = __fdiv_rn(ss, (float)size);
  ss = __fadd_rn(ss, eps);
  return __fdiv_rn(1.0f, __fsqrt_rn(ss));
}

// One normalized value: weight * (inv * x), the reference's rounding steps.
__device__ __forceinline__ float rms_apply(float x, float w, float inv) { return __fmul_rn(w, __fmul_rn(inv, x)); }

// k_quantize's per-value rule (src/gemv.c:617-621): q = (int8)roundf(clamp(x / scale, -127, 127)), 0 when scale == 0.
__device__ __forceinline__ int quantize_value(float x, float scale) {
  float v = scale == 0.0f ? 0.0f : __fdiv_rn(x, scale);
  v = fmaxf(-127.0f, fminf(127.0f, v));
  return (int)roundf(v);
}
