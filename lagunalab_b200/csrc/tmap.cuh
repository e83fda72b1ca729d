// Host-side TMA tensor-map encoding (cuTensorMapEncodeTiled through the runtime's driver
// entry point, so the library links only cudart).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace lg {

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2D row-major map: `rows` rows of `inner` elements (bf16 or uint32), `row_bytes` apart; a
// box of box_inner x box_rows; swz = 128 / 32 / 0 for the 128-byte, 32-byte or no swizzle.
// Rows past `rows` read as zeros.
inline int make_map_2d(CUtensorMap* m, const void* base, bool bf16, uint64_t inner,
                       uint64_t rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows,
                       int swz) {
  auto fn = tmap_encode_fn();
  if (!fn) return fail(LG_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                             : (swz == 32 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE),
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LG_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LG_OK;
}

}  // namespace lg
