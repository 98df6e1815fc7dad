// decode_e2e.cpp -- the decode step end to end through the C++ drop-in header.
//
// What a C++ caller of alpaka::nn::onHost writes for one decode step of the
// attention path, with host buffers: copy this step's query rows, new key rows
// and hidden states from (pinned) host memory, rmsNorm the hidden states,
// ropeInPlace Q and the new K row at position Tk, fused decode attention over
// this rank's KV cache slice -- on N > 1 ranks through the multicast output
// (attentionDecodeMirror) and the signal barrier -- and copy the full output
// back. bench.py times `steps` such steps with CUDA events on the caller's
// stream (its `e2e` figure); the library is built beside the drop-in test
// program by tests/cpp/build.py.
#include <cuda_runtime.h>

#include <cstdint>
#include <exception>
#include <string>

#include "alpakann_b200/onHost.hpp"

namespace {
thread_local std::string g_error;
}

extern "C" {

struct DecodeE2E {
    int32_t B, Hl, H, Tk, D, dm;  // batch, local / total heads, cache length, head dim, d_model
    float eps, scale;
    uint32_t position;
    // pinned host buffers
    float const* h_q;       // [B,1,Hl,D]
    float const* h_knew;    // [B,1,Hl,D]
    float const* h_hidden;  // [B,dm]
    float* h_out;           // [B,1,H,D]
    // device buffers
    float* q;
    float* knew;
    float* hidden;
    float* normed;
    float const* norm_w;  // [dm]
    float const* cos_t;   // [Tk+1, D/2]
    float const* sin_t;
    float const* const* k_caches;  // n_caches copies of [B,Hl,Tk,D]; step i reads copy i % n_caches
    float const* const* v_caches;
    int32_t n_caches;
    float* out;       // [B,1,H,D]; this rank's heads start at head `head0`
    int32_t head0;
    // multicast gather (nranks > 1): mirror of out[.., head0, ..] and the barrier's signals
    void* out_mirror;
    uint32_t* signals;
    uint32_t* const* peer_signals;
    int32_t nranks, rank;
    uint32_t* epoch_word;  // this rank's barrier epoch, in device memory
    uint64_t timeout_ns;
};

const char* decode_e2e_error(void) { return g_error.c_str(); }

// Runs `steps` steps on `stream`; *ms = device time between events around them.
int decode_e2e_run(DecodeE2E* a, int steps, cudaStream_t stream, float* ms) {
    namespace b2 = alpaka::nn::b200;
    namespace nn = alpaka::nn::onHost::nn;
    try {
        int dev = 0;
        cudaGetDevice(&dev);
        b2::Queue queue(stream, dev);
        int64_t const B = a->B, Hl = a->Hl, H = a->H, D = a->D, dm = a->dm;
        auto vq = b2::makeView<float, 4>(a->q, {B, 1, Hl, D});
        auto vkn = b2::makeView<float, 4>(a->knew, {B, 1, Hl, D});
        auto vh = b2::makeView<float, 2>(a->hidden, {B, dm});
        auto vn = b2::makeView<float, 2>(a->normed, {B, dm});
        auto vw = b2::makeView<float const, 1>(a->norm_w, {dm});
        auto vcos = b2::makeView<float const, 2>(a->cos_t, {static_cast<int64_t>(a->Tk) + 1, D / 2});
        auto vsin = b2::makeView<float const, 2>(a->sin_t, {static_cast<int64_t>(a->Tk) + 1, D / 2});
        // this rank's heads of the full output: a strided view
        auto full = b2::makeView<float, 4>(a->out, {B, 1, H, D});
        auto vout = b2::subView<float, 4>(full, {0, 0, a->head0, 0}, {B, 1, Hl, D});
        size_t const qb = static_cast<size_t>(B * Hl * D) * sizeof(float);
        size_t const hb = static_cast<size_t>(B * dm) * sizeof(float);
        size_t const ob = static_cast<size_t>(B * H * D) * sizeof(float);
        cudaEvent_t e0, e1;
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaEventRecord(e0, stream);
        for (int i = 0; i < steps; ++i) {
            cudaMemcpyAsync(a->q, a->h_q, qb, cudaMemcpyHostToDevice, stream);
            cudaMemcpyAsync(a->knew, a->h_knew, qb, cudaMemcpyHostToDevice, stream);
            cudaMemcpyAsync(a->hidden, a->h_hidden, hb, cudaMemcpyHostToDevice, stream);
            nn::rmsNorm<float>(queue, 0, vh, vw, vn, a->eps);
            nn::ropeInPlace<float>(queue, 0, vq, vkn, vcos, vsin, alpaka::nn::RopeLayout::BTHD, a->position);
            int const c = i % a->n_caches;
            auto vk = b2::makeView<float const, 4>(a->k_caches[c], {B, Hl, a->Tk, D});
            auto vv = b2::makeView<float const, 4>(a->v_caches[c], {B, Hl, a->Tk, D});
            if (a->nranks == 1) {
                nn::attentionDecode<float>(queue, 0, vq, vk, vv, vout, a->scale, 1u, alpaka::nn::AttentionKvLayout::BHTD);
            } else {
                nn::attentionDecodeMirror<float>(queue, 0, vq, vk, vv, vout, a->out_mirror, a->scale, 1u,
                                                 alpaka::nn::AttentionKvLayout::BHTD);
                b2::signalBarrierDev(queue, a->signals, a->peer_signals, a->nranks, a->rank, a->epoch_word,
                                     a->timeout_ns);
            }
            cudaMemcpyAsync(a->h_out, a->out, ob, cudaMemcpyDeviceToHost, stream);
        }
        cudaEventRecord(e1, stream);
        cudaError_t const err = cudaEventSynchronize(e1);
        cudaEventElapsedTime(ms, e0, e1);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        if (err != cudaSuccess) {
            g_error = cudaGetErrorString(err);
            return 2;
        }
        return 0;
    } catch (std::exception const& e) {
        g_error = e.what();
        return 1;
    }
}

}  // extern "C"
