// selftest.cu -- exercises the failure-detection path every kernel with a wait
// shares: a bounded mbarrier wait that gives up, sets a bit in a device error
// word, and returns, leaving the context usable.
//
// One CTA initialises an mbarrier for one arrival and waits on it with
// mbar_wait_bounded (the helper the decode and prefill kernels use). With
// `arrive` set, thread 0 arrives first and the wait completes at once; without
// it nothing ever arrives, the wait gives up after `limit_ns`, and
// ANN_DEVERR_WAIT_TIMEOUT is reported through ann_take_device_error.
#include "common.cuh"
#include "tma.cuh"

namespace ann {

int take_selftest_error(cudaStream_t s, uint32_t* bits);

namespace {

__device__ unsigned int g_selftest_error;

__global__ void __launch_bounds__(32) wait_probe_kernel(uint64_t limit_ns, int arrive) {
    __shared__ __align__(8) uint64_t bar_storage;
    uint32_t const bar = smem_u32(&bar_storage);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (arrive && threadIdx.x == 0) mbar_arrive(bar);
    bool const ok = mbar_wait_bounded(bar, 0, limit_ns);
    if (!ok && threadIdx.x == 0) atomicOr(&g_selftest_error, ANN_DEVERR_WAIT_TIMEOUT);
}

}  // namespace

int take_selftest_error(cudaStream_t s, uint32_t* bits) {
    unsigned int value = 0, zero = 0;
    if (cudaMemcpyFromSymbolAsync(&value, g_selftest_error, sizeof value, 0, cudaMemcpyDeviceToHost, s) !=
            cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_selftest_error, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ANN_ECUDA, "device error word: %s", cudaGetErrorString(cudaGetLastError()));
    *bits |= value;
    return ANN_OK;
}

}  // namespace ann

extern "C" int ann_selftest_wait(ann_stream stream, int32_t arrive, uint64_t limit_ns) {
    ANN_API_BEGIN
    if (limit_ns > 2000000000ull) return ann::fail(ANN_EINVAL, "selftest: limit_ns above 2 s.");
    ann::wait_probe_kernel<<<1, 32, 0, ann::as_stream(stream)>>>(limit_ns, arrive ? 1 : 0);
    return ann::check_launch("selftest wait");
    ANN_API_END
}
