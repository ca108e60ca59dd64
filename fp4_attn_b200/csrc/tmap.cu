// tmap.cu -- cuTensorMapEncodeTiled through cudaGetDriverEntryPoint.
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "status.h"
#include "tmap.h"

namespace fp4 {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int encode_tiled_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t dim0, uint64_t dim1,
                    uint64_t row_stride_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return set_error(FP4ATTN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (no CUDA driver?)");
  cuuint64_t dims[2] = {dim0, dim1};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box0, box1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FP4ATTN_OK : set_error(FP4ATTN_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
}

}  // namespace fp4
