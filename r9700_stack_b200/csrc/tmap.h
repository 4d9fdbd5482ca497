// Host-side TMA tensor-map construction (cuTensorMapEncodeTiled through the runtime's driver
// entry point, so the extension does not link libcuda directly). Every map here is 2-D, K-major
// (the contiguous dimension is the reduction dimension) and uses the 128-byte swizzle that the
// UMMA K-major SW128 descriptor expects.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <cstdint>

namespace r9k {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && p != nullptr, "r9k: cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

inline CUtensorMap make_tmap_2d(CUtensorMapDataType dt, void* base, uint64_t inner, uint64_t outer,
                                uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                                CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "r9k: cuTensorMapEncodeTiled failed (", (int)r, ") dt=", (int)dt, " inner=", inner,
              " outer=", outer, " stride=", row_stride_bytes, " box=", box_inner, "x", box_outer);
  return m;
}

// packed e2m1 rows [rows, K/2 bytes] landing in smem as 16U4_ALIGN16B (1 byte per element)
inline CUtensorMap tmap_fp4_kmajor(void* base, int64_t rows, int64_t K, int box_rows) {
  TORCH_CHECK(K % 128 == 0, "fp4 tensor map: K must be a multiple of 128");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 31) == 0, "fp4 tensor map: base must be 32-byte aligned");
  return make_tmap_2d(CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, base, (uint64_t)K, (uint64_t)rows, (uint64_t)(K / 2), 128,
                      (uint32_t)box_rows);
}
inline CUtensorMap tmap_u8_kmajor(void* base, int64_t rows, int64_t K, int box_rows, int64_t ld = -1) {
  if (ld < 0) ld = K;
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0 && ld % 16 == 0, "u8 tensor map: 16-byte alignment");
  return make_tmap_2d(CU_TENSOR_MAP_DATA_TYPE_UINT8, base, (uint64_t)K, (uint64_t)rows, (uint64_t)ld, 128,
                      (uint32_t)box_rows);
}
inline CUtensorMap tmap_bf16_kmajor(void* base, int64_t rows, int64_t K, int64_t ld, int box_rows) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0 && (ld * 2) % 16 == 0, "bf16 tensor map: alignment");
  return make_tmap_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, (uint64_t)K, (uint64_t)rows, (uint64_t)(ld * 2), 64,
                      (uint32_t)box_rows);
}

// Packed fp4 weights read as plain bytes (expanded on chip): box of 128 rows x 64 bytes, no swizzle.
inline CUtensorMap tmap_fp4_packed(void* base, int64_t rows, int64_t K) {
  return make_tmap_2d(CU_TENSOR_MAP_DATA_TYPE_UINT8, base, (uint64_t)(K / 2), (uint64_t)rows, (uint64_t)(K / 2), 64, 128,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
}
inline CUtensorMap tmap_units_packed_3d(void* base, int64_t units) {
  CUtensorMap m;
  cuuint64_t dims[3] = {64, 128, (cuuint64_t)units};
  cuuint64_t strides[2] = {64, 64 * 128};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "r9k: packed tiled weight tensor map failed (", (int)r, ")");
  return m;
}

// Pre-tiled weights: [units][128 rows][row_bytes] with every unit (128 rows x 128 K elements)
// contiguous, so one TMA box is one contiguous 8 KB (fp4) / 16 KB (fp8) read from HBM.
inline CUtensorMap tmap_units_3d(void* base, int64_t units, bool fp4) {
  const uint64_t row_bytes = fp4 ? 64 : 128;
  CUtensorMap m;
  cuuint64_t dims[3] = {128, 128, (cuuint64_t)units};
  cuuint64_t strides[2] = {row_bytes, row_bytes * 128};
  cuuint32_t box[3] = {128, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 31) == 0, "tiled weight: base must be 32-byte aligned");
  CUresult r = get_encode_fn()(&m, fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base,
                               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "r9k: tiled weight tensor map failed (", (int)r, ")");
  return m;
}

}  // namespace r9k
