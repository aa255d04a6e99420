// hb_tma.cu -- tensor-map encoding for the TMA copies of every kernel
// (cuTensorMapEncodeTiled, reached through the runtime's driver entry point
// so the library needs no link-time libcuda symbol).
#include <cuda.h>
#include <cuda_runtime.h>

#include "hb_internal.h"

namespace hb {
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

}  // namespace

bool encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                  const cuuint64_t* dims, const cuuint64_t* strides_bytes, const cuuint32_t* box,
                  CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return fn(map, dt, cuuint32_t(rank), const_cast<void*>(base), dims, strides_bytes, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* base,
               uint64_t rows, uint64_t cols, uint64_t row_stride_elems, uint32_t box_rows,
               uint32_t box_cols, CUtensorMapSwizzle swizzle) {
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride_elems * uint64_t(elem_bytes)};
  const cuuint32_t box[2] = {box_cols, box_rows};
  return encode_tiled(map, dt, 2, base, dims, strides, box, swizzle);
}

}  // namespace hb
