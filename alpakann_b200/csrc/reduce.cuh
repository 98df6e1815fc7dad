// reduce.cuh -- warp / block reductions and precision-matched math helpers.
#pragma once

#include <cuda_runtime.h>

#include <cfloat>

namespace ann {

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide reductions for blockDim.x == 32 * NW threads. `scratch` holds NW
// values; every thread gets the result. Contains two __syncthreads().
template <int NW, typename T>
__device__ __forceinline__ T block_sum(T v, T* scratch) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
    __syncthreads();
    T r = scratch[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) r += scratch[w];
    __syncthreads();
    return r;
}

template <int NW, typename T>
__device__ __forceinline__ T block_max(T v, T* scratch) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
    __syncthreads();
    T r = scratch[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) r = fmax(r, scratch[w]);
    __syncthreads();
    return r;
}

template <typename T>
struct Lowest;
template <>
struct Lowest<float> {
    static constexpr float value = -FLT_MAX;
};
template <>
struct Lowest<double> {
    static constexpr double value = -DBL_MAX;
};

// -infinity of T (exp of it is exactly 0).
__device__ __forceinline__ float neg_inf(float) { return __int_as_float(0xff800000); }
__device__ __forceinline__ double neg_inf(double) { return __longlong_as_double(static_cast<long long>(0xfff0000000000000ull)); }

// 1/sqrt: rsqrtf for fp32 (within 2 ulp), correctly rounded sqrt and divide
// for fp64 so the 1e-11 budget is not spent here.
__device__ __forceinline__ float rsqrt_t(float x) { return rsqrtf(x); }
__device__ __forceinline__ double rsqrt_t(double x) { return 1.0 / sqrt(x); }

__device__ __forceinline__ float exp_t(float x) { return expf(x); }
__device__ __forceinline__ double exp_t(double x) { return exp(x); }

// Uncontracted products/sums (no FMA), so results are bit-identical to a host
// loop compiled without FP contraction.
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }

}  // namespace ann
