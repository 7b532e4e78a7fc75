// TMA tensor-map construction shared by the tensor-core kernels.
//
// cuTensorMapEncodeTiled is a driver entry point; it is looked up once
// through the runtime (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace b2k {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
  }();
  return fn;
}

// Row-major FP32 matrix [rows][inner] with a row stride of `ld` elements,
// copied in boxes of box_rows x box_inner with the given shared-memory
// swizzle.  Elements outside the matrix read as zero.  Requires a 16-byte
// aligned base and ld * 4 a multiple of 16.
inline int make_map_2d(b2k_ctx *ctx, CUtensorMap *map, const float *base, int64_t inner, int64_t rows, int64_t ld,
                       uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  auto encode = tensor_map_encoder();
  if (!encode) return fail(ctx, B2K_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult res = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) return fail(ctx, B2K_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)res);
  return B2K_OK;
}

}  // namespace b2k
