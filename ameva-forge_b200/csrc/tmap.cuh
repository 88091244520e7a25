// Host-side TMA tensor-map encoding (cuTensorMapEncodeTiled resolved through
// the runtime's driver entry point, so the library does not link libcuda)
// and the device-side tiled bulk-tensor load.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace fg {

// 2-D row-major tensor [rows][cols] of `elem_bytes`-byte elements with a row
// pitch of `pitch_bytes`, tiled in boxes of box_rows x box_cols elements; no
// swizzle, out-of-bounds elements read as zero.  Requirements checked here:
// base 16-byte aligned, pitch a multiple of 16, box_cols * elem_bytes a
// multiple of 16.
// `swizzle` other than NONE lays the box out in shared memory with that
// swizzle (the destination must then be 1024-byte aligned and box_cols *
// elem_bytes at most the swizzle span).
CUtensorMap make_tmap_2d(const void *base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows, uint64_t cols,
                         uint64_t pitch_bytes, uint32_t box_rows, uint32_t box_cols,
                         CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE);

// 3-D tensor [d2][d1][d0] of `elem_bytes`-byte elements (d0 contiguous, strides
// s1 and s2 in bytes, multiples of 16, in any order), tiled in boxes
// b0 x b1 x b2 laid out densely in shared memory as [b2][b1][b0] rows of
// b0 elements (swizzled like a 2-D box of b1 * b2 rows when `swizzle` is
// not NONE); out-of-bounds elements read as zero.
CUtensorMap make_tmap_3d(const void *base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0, uint64_t d1,
                         uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2,
                         CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE);

// 4-D tensor [d3][d2][d1][d0] (d0 contiguous; strides s1..s3 in bytes,
// multiples of 16), boxes b0 x b1 x b2 x b3 laid out densely as
// [b3][b2][b1][b0], swizzled like a 2-D box of b1 * b2 * b3 rows.
CUtensorMap make_tmap_4d(const void *base, CUtensorMapDataType dtype, int elem_bytes, const uint64_t (&dims)[4],
                         const uint64_t (&strides)[3], const uint32_t (&box)[4],
                         CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE);

// Tiled 2-D load of the box at (x = column, y = row) into shared memory,
// completing on `bar`.  x * elem_bytes must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int32_t x, int32_t y, uint64_t *bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"((uint32_t)__cvta_generic_to_shared(bar)), "l"(policy)
      : "memory");
}

// Tiled 3-D load of the box at (x, y, z); x * elem_bytes must be a multiple of 16.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int32_t x, int32_t y, int32_t z,
                                            uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"((uint32_t)__cvta_generic_to_shared(bar)),
      "l"(policy)
      : "memory");
}

// Tiled 4-D load of the box at (x, y, z, w); x * elem_bytes must be a multiple of 16.
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int32_t x, int32_t y, int32_t z,
                                            int32_t w, uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w),
      "r"((uint32_t)__cvta_generic_to_shared(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace fg
