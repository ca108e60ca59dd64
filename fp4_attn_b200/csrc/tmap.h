// tmap.h -- TMA tensor-map encoding without a link-time libcuda dependency
// (the driver entry point is resolved through the runtime on first use, so
// the library still loads on machines without a GPU driver).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace fp4 {
// 2-D tiled map: dim0 (innermost, elements) x dim1 rows, row stride in bytes.
int encode_tiled_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t dim0, uint64_t dim1,
                    uint64_t row_stride_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle);
}  // namespace fp4
