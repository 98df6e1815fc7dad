// multicast.cu -- the cross-rank barrier that publishes multicast ("mirror") outputs.
//
// The head-sharded path gathers per-rank outputs without a collective: the
// decode and prefill kernels of every rank store their head slices through an
// NVLink multicast address into every rank's copy of the full output
// (multimem.st, csrc/multimem.cuh). What remains is to know that all ranks
// have finished: this barrier. Every rank holds an array of nranks 32-bit
// signal words, and every rank can address every rank's array (peer mappings
// over NVLink, e.g. torch symmetric memory's buffer pointers). Enqueued on a
// stream, after the producing kernel, the barrier kernel
//   1. fences at system scope, then stores the call's epoch into word `rank`
//      of every rank's array (a release store at system scope per rank);
//   2. waits until every word of its own array holds that epoch (or a later
//      one), with acquire loads at system scope.
// ann_signal_barrier_dev takes the epoch from a word in this rank's device
// memory instead (the previous epoch + 1, written back by the kernel), so that a
// captured CUDA graph that replays it runs a new epoch every time.
// Every wait is bounded: after `timeout_ns` the kernel sets
// ANN_DEVERR_WAIT_TIMEOUT in its device error word and returns, so a rank that
// left leaves the others with an error status, not a hung GPU. The barrier
// itself issues plain stores only (no multimem, no loads from peer memory).
#include "common.cuh"
#include "tma.cuh"

namespace ann {

int take_multicast_error(cudaStream_t s, uint32_t* bits);

namespace {

__device__ unsigned int g_mc_error;

constexpr int kMaxRanks = 32;

// epoch_word != null: the epoch is *epoch_word + 1 (0 skipped), stored back at the end
__global__ void __launch_bounds__(32) mc_barrier_kernel(uint32_t* signals, uint32_t* const* peer_signals, int nranks,
                                                        int rank, uint32_t epoch, uint32_t* epoch_word,
                                                        uint64_t limit_ns) {
    int const t = threadIdx.x;
    if (epoch_word != nullptr) {
        epoch = *epoch_word + 1u;
        if (epoch == 0u) epoch = 1u;
    }
    if (t < nranks) {
        __threadfence_system();  // everything this stream wrote before is performed first
        uint32_t* const dst = peer_signals[t] + rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst), "r"(epoch) : "memory");
        uint64_t const t0 = global_timer_ns();
        for (;;) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(signals + t) : "memory");
            if (static_cast<int32_t>(v - epoch) >= 0) break;
            if (global_timer_ns() - t0 > limit_ns) {
                atomicOr(&g_mc_error, ANN_DEVERR_WAIT_TIMEOUT);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncwarp();  // every lane has read the old epoch word
    if (t == 0 && epoch_word != nullptr) *epoch_word = epoch;
}

}  // namespace

int take_multicast_error(cudaStream_t s, uint32_t* bits) {
    unsigned int value = 0, zero = 0;
    if (cudaMemcpyFromSymbolAsync(&value, g_mc_error, sizeof value, 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_mc_error, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ANN_ECUDA, "device error word: %s", cudaGetErrorString(cudaGetLastError()));
    *bits |= value;
    return ANN_OK;
}

}  // namespace ann

extern "C" int ann_signal_barrier(ann_stream stream, uint32_t* signals, uint32_t* const* peer_signals,
                                  int32_t nranks, int32_t rank, uint32_t epoch, uint64_t timeout_ns) {
    ANN_API_BEGIN
    using namespace ann;
    if (signals == nullptr || peer_signals == nullptr) return fail(ANN_EINVAL, "signal barrier: NULL signals.");
    if (!aligned(signals, 4) || !aligned(peer_signals, 8))
        return fail(ANN_EINVAL, "signal barrier: misaligned signals.");
    if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
        return fail(ANN_EINVAL, "signal barrier: rank %d of %d ranks (at most %d).", static_cast<int>(rank),
                    static_cast<int>(nranks), kMaxRanks);
    if (epoch == 0u) return fail(ANN_EINVAL, "signal barrier: epochs start at 1 (the signals start at 0).");
    if (timeout_ns == 0 || timeout_ns > 60000000000ull)
        return fail(ANN_EINVAL, "signal barrier: timeout must be in (0, 60 s].");
    mc_barrier_kernel<<<1, 32, 0, as_stream(stream)>>>(signals, peer_signals, nranks, rank, epoch, nullptr,
                                                       timeout_ns);
    return check_launch("signal barrier");
    ANN_API_END
}

extern "C" int ann_signal_barrier_dev(ann_stream stream, uint32_t* signals, uint32_t* const* peer_signals,
                                      int32_t nranks, int32_t rank, uint32_t* epoch_word, uint64_t timeout_ns) {
    ANN_API_BEGIN
    using namespace ann;
    if (signals == nullptr || peer_signals == nullptr || epoch_word == nullptr)
        return fail(ANN_EINVAL, "signal barrier: NULL signals or epoch word.");
    if (!aligned(signals, 4) || !aligned(peer_signals, 8) || !aligned(epoch_word, 4))
        return fail(ANN_EINVAL, "signal barrier: misaligned signals.");
    if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
        return fail(ANN_EINVAL, "signal barrier: rank %d of %d ranks (at most %d).", static_cast<int>(rank),
                    static_cast<int>(nranks), kMaxRanks);
    if (timeout_ns == 0 || timeout_ns > 60000000000ull)
        return fail(ANN_EINVAL, "signal barrier: timeout must be in (0, 60 s].");
    mc_barrier_kernel<<<1, 32, 0, as_stream(stream)>>>(signals, peer_signals, nranks, rank, 0u, epoch_word,
                                                       timeout_ns);
    return check_launch("signal barrier");
    ANN_API_END
}
