// Host-side TMA tensor maps (cuTensorMapEncodeTiled) for the weight and scale matrices, cached per (address, shape,
// box): encoding costs microseconds of host time, and the same weights are used every decode step.
#pragma once

#include <cuda.h>
#include <stdint.h>

// 2-D row-major matrix [rows][cols] of `elem_bytes`-byte elements with row stride `ld_bytes`; boxes of
// box_cols x box_rows elements; swizzle128 selects the 128-byte swizzle (box_cols * elem_bytes must then be <= 128).
// Returns false (and leaves *out untouched) if the driver refuses the shape.
bool kc_tmap_2d(CUtensorMap *out, const void *base, int elem_bytes, uint64_t cols, uint64_t rows, uint64_t ld_bytes,
                uint32_t box_cols, uint32_t box_rows, bool swizzle128);

// int8 matrix [rows][k] (row stride ld bytes, k % 128 == 0) viewed as [k / 128][rows][128] (strides 128 B and ld):
// one box of box_kb x box_rows x 128 B lands in shared memory as box_kb blocks of [box_rows][128 B], 128B-swizzled,
// i.e. a whole [box_rows x box_kb*128 B] tile in one TMA instruction.
bool kc_tmap_kblocks(CUtensorMap *out, const void *base, uint64_t k, uint64_t rows, uint64_t ld_bytes, uint32_t box_kb,
                     uint32_t box_rows);
