#include <cudaTypedefs.h>

#include <mutex>

#include "tmap.cuh"

namespace fg {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    cudaGetLastError();
  });
  FG_REQUIRE(fn != nullptr, FG_ERR_UNAVAILABLE, "cuTensorMapEncodeTiled is not available from the driver");
  return fn;
}
}  // namespace

CUtensorMap make_tmap_2d(const void *base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows, uint64_t cols,
                         uint64_t pitch_bytes, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swizzle) {
  FG_REQUIRE(((uintptr_t)base & 15) == 0 && pitch_bytes % 16 == 0 && (box_cols * elem_bytes) % 16 == 0 &&
                 box_rows >= 1 && box_rows <= 256 && box_cols >= 1 && box_cols <= 256,
             FG_ERR_VALIDATION, "tensor map: misaligned base/pitch/box");
  CUtensorMap m;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {pitch_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FG_REQUIRE(r == CUDA_SUCCESS, FG_ERR_INTERNAL_GPU, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return m;
}

CUtensorMap make_tmap_3d(const void *base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0, uint64_t d1,
                         uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2,
                         CUtensorMapSwizzle swizzle) {
  FG_REQUIRE(((uintptr_t)base & 15) == 0 && s1 % 16 == 0 && s2 % 16 == 0 && (b0 * elem_bytes) % 16 == 0 &&
                 b0 >= 1 && b0 <= 256 && b1 >= 1 && b1 <= 256 && b2 >= 1 && b2 <= 256,
             FG_ERR_VALIDATION, "tensor map: misaligned base/stride/box");
  CUtensorMap m;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {s1, s2};
  const cuuint32_t box[3] = {b0, b1, b2};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, dtype, 3, const_cast<void *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FG_REQUIRE(r == CUDA_SUCCESS, FG_ERR_INTERNAL_GPU, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return m;
}

CUtensorMap make_tmap_4d(const void *base, CUtensorMapDataType dtype, int elem_bytes, const uint64_t (&dims)[4],
                         const uint64_t (&strides)[3], const uint32_t (&box)[4], CUtensorMapSwizzle swizzle) {
  bool ok = ((uintptr_t)base & 15) == 0 && (box[0] * elem_bytes) % 16 == 0;
  for (int i = 0; i < 3; ++i) ok = ok && strides[i] % 16 == 0;
  for (int i = 0; i < 4; ++i) ok = ok && box[i] >= 1 && box[i] <= 256 && dims[i] >= 1;
  FG_REQUIRE(ok, FG_ERR_VALIDATION, "tensor map: misaligned base/stride/box");
  CUtensorMap m;
  const cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  const cuuint64_t st[3] = {strides[0], strides[1], strides[2]};
  const cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(&m, dtype, 4, const_cast<void *>(base), d, st, bx, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FG_REQUIRE(r == CUDA_SUCCESS, FG_ERR_INTERNAL_GPU, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return m;
}

}  // namespace fg
