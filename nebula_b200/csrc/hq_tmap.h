// hq_tmap.h -- host-side creation of TMA tensor maps (cuTensorMapEncodeTiled),
// fetched through cudaGetDriverEntryPoint so the library needs no libcuda link.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hq {

// 2-D row-major tensor [outer][inner] of `dt` elements, rows `row_bytes` apart
// (a multiple of 16), box [box_outer][box_inner]; out-of-range boxes read zeros.
cudaError_t make_tmap_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dt, uint64_t inner,
                         uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle);

}  // namespace hq
