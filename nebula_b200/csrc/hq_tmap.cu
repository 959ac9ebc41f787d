// hq_tmap.cu -- TMA tensor-map encoding (see hq_tmap.h).
#include "hq_tmap.h"

#include <cudaTypedefs.h>

#include <mutex>

namespace hq {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}
}  // namespace

cudaError_t make_tmap_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dt, uint64_t inner,
                         uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estride[2] = {1, 1};
    CUresult r = fn(out, dt, 2, const_cast<void*>(base), dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace hq
