// Inline-PTX wrappers for the 5th-generation tensor core (tcgen05) and tensor memory (TMEM) on sm_100a.
// Descriptor formats follow the PTX ISA: shared-memory matrix descriptor (start address >> 4 in bits 0-13, leading
// byte offset >> 4 in 16-29, stride byte offset >> 4 in 32-45, version 1 in 46-47, layout type in 61-63) and the
// instruction descriptor of kind::i8 (accumulator format in bits 4-5, A/B formats in 7-9 / 10-12, K-major bits 15/16,
// N >> 3 in 17-22, M >> 4 in 24-28).
#pragma once

#include <stdint.h>

#include "common.cuh"

// K-major operand tile in the canonical 128-byte-swizzle layout: 8-row x 128 B atoms stacked along M/N (1024 B apart).
__device__ __forceinline__ uint64_t umma_desc_sw128(const void *smem_tile) {
  const uint64_t addr = smem_u32(smem_tile);
  uint64_t d = (addr >> 4) & 0x3FFFull;       // start address
  d |= (uint64_t)1 << 16;                      // leading byte offset (unused for swizzled K-major): 16 B
  d |= (uint64_t)(1024 >> 4) << 32;            // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                      // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                      // SWIZZLE_128B
  return d;
}

// Non-swizzled K-major layout (8-row x 16-byte core matrices): leading / stride byte offsets between core matrices.
__device__ __forceinline__ uint64_t umma_desc_plain(const void *smem_tile, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  const uint64_t addr = smem_u32(smem_tile);
  uint64_t d = (addr >> 4) & 0x3FFFull;
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  return d;  // layout type 0: no swizzle
}

// Copies 128 lanes x 256 bits (8 columns) from shared memory into TMEM, in the tensor pipe's issue order (it is
// implicitly pipelined with the same thread's later tcgen05.mma).
__device__ __forceinline__ void tmem_cp_128x256b(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// kind::i8 instruction descriptor: signed int8 A and B, both K-major, int32 accumulators, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}

// The mbarrier tracks completion of every tcgen05 operation this thread issued before it.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes (this warp's quadrant) x 32 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes (this warp's quadrant) x 32 consecutive 32-bit columns, as 16 packed pairs of neighbouring columns (the
// operand form of the f32x2 instructions: no register moves between the load and packed arithmetic).
__device__ __forceinline__ void tmem_ld32_pairs(uint32_t taddr, uint64_t (&r)[16]) {
  asm volatile(
      "{\n\t.reg .b32 a0, a1, a2, a3, a4, a5, a6, a7, a8, a9, a10, a11, a12, a13, a14, a15;\n\t"
      ".reg .b32 a16, a17, a18, a19, a20, a21, a22, a23, a24, a25, a26, a27, a28, a29, a30, a31;\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {a0, a1, a2, a3, a4, a5, a6, a7, a8, a9, a10, a11, a12, a13, a14, a15,"
      " a16, a17, a18, a19, a20, a21, a22, a23, a24, a25, a26, a27, a28, a29, a30, a31}, [%16];\n\t"
      "mov.b64 %0, {a0, a1};\n\t"
      "mov.b64 %1, {a2, a3};\n\t"
      "mov.b64 %2, {a4, a5};\n\t"
      "mov.b64 %3, {a6, a7};\n\t"
      "mov.b64 %4, {a8, a9};\n\t"
      "mov.b64 %5, {a10, a11};\n\t"
      "mov.b64 %6, {a12, a13};\n\t"
      "mov.b64 %7, {a14, a15};\n\t"
      "mov.b64 %8, {a16, a17};\n\t"
      "mov.b64 %9, {a18, a19};\n\t"
      "mov.b64 %10, {a20, a21};\n\t"
      "mov.b64 %11, {a22, a23};\n\t"
      "mov.b64 %12, {a24, a25};\n\t"
      "mov.b64 %13, {a26, a27};\n\t"
      "mov.b64 %14, {a28, a29};\n\t"
      "mov.b64 %15, {a30, a31};\n\t"
      "}"
      : "=l"(r[0]), "=l"(r[1]), "=l"(r[2]), "=l"(r[3]), "=l"(r[4]), "=l"(r[5]), "=l"(r[6]), "=l"(r[7]),
        "=l"(r[8]), "=l"(r[9]), "=l"(r[10]), "=l"(r[11]), "=l"(r[12]), "=l"(r[13]), "=l"(r[14]), "=l"(r[15])
      : "r"(taddr));
}

// 32 lanes (this warp's quadrant) x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Writes the same 32-bit value into 32 lanes x 32 columns.
__device__ __forceinline__ void tmem_st32_fill(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
      "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
      "r"(v)
      : "memory");
}

// Packed fp32x2 arithmetic (each lane rounded exactly like the scalar instruction).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t f2_pack_bits(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
