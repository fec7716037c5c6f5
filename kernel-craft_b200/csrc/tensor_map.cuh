// tensor_map.cuh -- host-side encoding of 2-D TMA tensor maps.
//
// cuTensorMapEncodeTiled is fetched from the driver at first use through
// cudaGetDriverEntryPoint, so the library has no link-time dependency on
// libcuda and still loads on machines without a GPU driver.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "kc_common.cuh"

namespace kc {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// Row-major 2-D tensor [outer][inner] of `elem_bytes`-byte elements with a row
// pitch of `row_bytes`; boxes of box_inner x box_outer elements.  Elements
// outside the tensor read as zero.  Returns KC_OK or a recorded error.
inline int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                     uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                     uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_tiled_fn();
    KC_REQUIRE(fn != nullptr, KC_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    KC_REQUIRE(r == CUDA_SUCCESS, KC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return KC_OK;
}

}  // namespace kc
