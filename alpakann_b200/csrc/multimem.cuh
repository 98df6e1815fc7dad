// multimem.cuh -- stores through an NVLink multicast address (NVSwitch NVLS), inline PTX.
//
// A multicast address maps one range that every rank of the node has bound
// to its own device memory; one multimem.st is replicated by the switch into
// every rank's copy (the issuing GPU's own copy included). The kernels that
// take an output "mirror" write their results this way, so the head-sharded
// outputs reach every rank inside the producing kernel, with no collective
// and no re-assembly pass. Only stores are issued here: there is no load or
// TMA copy from multicast or peer memory anywhere in this library.
#pragma once

#include <cstdint>

namespace ann::mc {

// 16 bytes (four 32-bit words; also used for two doubles' bits). addr 16-byte aligned.
__device__ __forceinline__ void store16(void* addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(__uint_as_float(a)),
                 "f"(__uint_as_float(b)), "f"(__uint_as_float(c)), "f"(__uint_as_float(d))
                 : "memory");
}
__device__ __forceinline__ void store(float* addr, float4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ void store(double* addr, double2 v) {
    uint64_t const x = static_cast<uint64_t>(__double_as_longlong(v.x)),
                   y = static_cast<uint64_t>(__double_as_longlong(v.y));
    store16(addr, static_cast<uint32_t>(x), static_cast<uint32_t>(x >> 32), static_cast<uint32_t>(y),
            static_cast<uint32_t>(y >> 32));
}
__device__ __forceinline__ void store(float* addr, float v) {
    asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void store(double* addr, double v) {
    asm volatile("multimem.st.relaxed.sys.global.f64 [%0], %1;" ::"l"(addr), "d"(v) : "memory");
}

// The element of the mirror at the same offset as `p` from `base`.
template <typename T>
__device__ __forceinline__ T* mirror_of(T* mirror, T const* base, T const* p) {
    return mirror + (p - base);
}

}  // namespace ann::mc
