// tmap.cuh -- host-side TMA tensor maps (cuTensorMapEncodeTiled) for the
// tensor-core kernels. The driver function is found through the runtime's
// entry-point query, so the library links no libcuda.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "common.cuh"

namespace ann {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled, or null when the driver does not offer it.
inline EncodeTiled encode_tiled() {
    static std::once_flag once;
    static EncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(f);
        else
            cudaGetLastError();
    });
    return fn;
}

// A rank-4 view [d3][d2][d1][d0] (d0 innermost, unit stride; element strides
// s[0..2] of d1..d3) that a tensor map can describe with 32-bit coordinates:
// every stride positive where its extent is above 1, element offsets below 2^36.
inline bool tma_view_ok(int64_t const (&dims)[4], int64_t const (&s)[3]) {
    for (int i = 0; i < 4; ++i)
        if (dims[i] < 1 || dims[i] + 256 > INT32_MAX) return false;
    for (int i = 0; i < 3; ++i)
        if ((s[i] <= 0 && dims[i + 1] > 1) || s[i] >= (int64_t{1} << 36)) return false;
    return s[0] * dims[1] < (int64_t{1} << 36) && s[1] * dims[2] < (int64_t{1} << 36) &&
           s[2] * dims[3] < (int64_t{1} << 36);
}

// fp32 tensor map over such a view with boxes of box0 x box1 x 1 x 1 elements
// and a 128-byte swizzle: 16-byte atoms (box0 = 32: piece j of box row r lands
// at r * 128 + ((j ^ (r % 8)) << 4) of a 1 KB-aligned box), or 32-byte atoms
// (CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B: 32-byte granule q of row r at
// r * 128 + ((q ^ (r % 4)) << 5)); elements outside the extents read as zero
// and are not written.
inline int map_f32_4d(CUtensorMap* map, const void* base, int64_t const (&dims)[4], int64_t const (&s)[3],
                      uint32_t box0, uint32_t box1, const char* what,
                      CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    EncodeTiled const enc = encode_tiled();
    if (enc == nullptr) return fail(ANN_ECUDA, "%s: cuTensorMapEncodeTiled is not available.", what);
    // the stride of a dimension of extent 1 is never used: give it a legal value
    int64_t const s1 = dims[1] == 1 ? (dims[0] + 3) / 4 * 4 : s[0];
    int64_t const s2 = dims[2] == 1 ? s1 * dims[1] : s[1];
    int64_t const s3 = dims[3] == 1 ? s2 * dims[2] : s[2];
    cuuint64_t const gdim[4] = {static_cast<cuuint64_t>(dims[0]), static_cast<cuuint64_t>(dims[1]),
                                static_cast<cuuint64_t>(dims[2]), static_cast<cuuint64_t>(dims[3])};
    cuuint64_t const gstr[3] = {static_cast<cuuint64_t>(s1) * 4, static_cast<cuuint64_t>(s2) * 4,
                                static_cast<cuuint64_t>(s3) * 4};
    cuuint32_t const box[4] = {box0, box1, 1, 1};
    cuuint32_t const unit[4] = {1, 1, 1, 1};
    CUresult const r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), gdim, gstr, box, unit,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ANN_ECUDA, "%s: cuTensorMapEncodeTiled failed (%d).", what, int(r));
    return ANN_OK;
}

}  // namespace ann
