// tmap.h -- host-side TMA tensor-map construction (driver entry point fetched
// through the runtime, so the extension does not link libcuda directly).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

namespace tmap {

using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                              const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                              const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeFn encoder() {
  static EncodeFn fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point unavailable");
    return reinterpret_cast<EncodeFn>(p);
  }();
  return fn;
}

// 2-D row-major tensor [rows, cols] of `elem_bytes` elements with row pitch
// `ld` elements; box [box_rows, box_cols]. Out-of-range boxes fill zeros.
inline CUtensorMap make_2d(const void *base, CUtensorMapDataType dtype, int elem_bytes,
                           uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                           uint32_t box_cols, CUtensorMapSwizzle swz,
                           CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  if ((ld * elem_bytes) % 16 != 0) throw std::runtime_error("TMA row pitch must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encoder()(&m, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swz, promo,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

// 4-D tensor, dims/box innermost first; byte strides of dims 1-3.
inline CUtensorMap make_4d(const void *base, CUtensorMapDataType dtype, const uint64_t (&dims)[4],
                           const uint64_t (&stride_bytes)[3], const uint32_t (&box)[4],
                           CUtensorMapSwizzle swz,
                           CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  for (uint64_t st : stride_bytes)
    if (st % 16 != 0) throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t st[3] = {stride_bytes[0], stride_bytes[1], stride_bytes[2]};
  cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encoder()(&m, dtype, 4, const_cast<void *>(base), d, st, bx, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swz, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled (4-D) failed: " + std::to_string((int)r));
  return m;
}

// 3-D tensor, dims/box innermost first; strides (bytes) of dims 1 and 2.
// Out-of-range boxes fill zeros.
inline CUtensorMap make_3d(const void *base, CUtensorMapDataType dtype, const uint64_t (&dims)[3],
                           const uint64_t (&stride_bytes)[2], const uint32_t (&box)[3],
                           CUtensorMapSwizzle swz,
                           CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  if (stride_bytes[0] % 16 != 0 || stride_bytes[1] % 16 != 0)
    throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t st[2] = {stride_bytes[0], stride_bytes[1]};
  cuuint32_t bx[3] = {box[0], box[1], box[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encoder()(&m, dtype, 3, const_cast<void *>(base), d, st, bx, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swz, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

// Paged KV cache [rows = pages * Hkv * 16, 128] bf16 (one page of one KV
// head = 16 contiguous rows of 256 bytes) as a 4-D map whose one box is a
// whole page-head (4 KB) in the 128-byte-swizzle layout the MMA descriptors
// read: dims (64 columns, 8 rows, 2 column halves, row groups of 8) with
// byte strides (256, 128, 2048); box (64, 8, 2, 2). In shared memory the
// box lands as [row group][half][8 rows][64 columns]: token t of a page
// block at (t / 8) * 2048 + half * 1024 + (t % 8) * 128, so 8-row atoms of
// one half sit 2048 bytes apart. Coordinate 3 is the row group (row / 8);
// a row group past the end reads zeros.
inline CUtensorMap make_kv_pages(const void *base, uint64_t rows, uint64_t row_bytes = 256) {
  if (rows % 8 != 0) throw std::runtime_error("paged KV rows must be a multiple of 8");
  return make_4d(base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, {64, 8, 2, rows / 8},
                 {row_bytes, 128, 8 * row_bytes}, {64, 8, 2, 2}, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace tmap
