// tma_host.h -- host-side creation of TMA tensor maps (cuTensorMapEncodeTiled through the
// runtime's driver entry point, so the library does not link libcuda directly).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "capi_internal.h"

namespace nvfp4 {

inline PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn() {
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

// 2D tensor [outer][inner] of `dtype` elements with a row pitch of `pitch_bytes`; box of
// box_inner x box_outer elements.  Out-of-range box elements read as zero.
inline nvfp4_status_t make_tmap_2d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dtype, int64_t inner,
                                   int64_t outer, int64_t pitch_bytes, int box_inner, int box_outer,
                                   CUtensorMapSwizzle swizzle) {
    auto enc = tma_encode_fn();
    if (!enc) return fail(NVFP4_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)pitch_bytes};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NVFP4_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return NVFP4_OK;
}

}  // namespace nvfp4
