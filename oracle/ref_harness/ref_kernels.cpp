// ref_kernels.cpp -- alpakaNN's own device kernels, run on the host.
//
// TEST INFRASTRUCTURE ONLY (built into oracle/_ref, never linked by the
// product). The reference's kernel sources are compiled UNMODIFIED from where
// they lie (-I <reference>/include) against the host-only alpaka stand-in in
// this directory, and each C entry point below applies one kernel functor to
// host views, exactly as the reference's onHost wrappers enqueue them:
//   AttentionScoresKernel / AttentionApplyKernel  onAcc/internal/nn/attention.hpp
//   EmbeddingLookupKernel                         onAcc/internal/nn/embedding.hpp
//   RmsNormKernel                                 onAcc/internal/nn/rms_norm.hpp
//   RopeSingleKernel                              onAcc/internal/nn/rope.hpp
//   SoftmaxKernel / MaskedSoftmaxKernel           onAcc/internal/nn/softmax.hpp
// The tests use these outputs to pin the CPU oracle (oracle/ann_oracle.cpp),
// which restates the same kernels, to the reference's own code.
#include <alpaka/nn/onAcc/internal/nn/attention.hpp>
#include <alpaka/nn/onAcc/internal/nn/embedding.hpp>
#include <alpaka/nn/onAcc/internal/nn/rms_norm.hpp>
#include <alpaka/nn/onAcc/internal/nn/rope.hpp>
#include <alpaka/nn/onAcc/internal/nn/softmax.hpp>

#include <cstdint>

namespace {

constexpr int kMaxRank = 8;

// The oracle's view descriptor (ann_view layout): data, rank, extents, BYTE pitches.
struct OView {
    void* data;
    int32_t rank;
    int32_t reserved;
    int64_t extents[kMaxRank];
    int64_t pitches[kMaxRank];
};

// A strided host view of rank N with alpaka's interface: getExtents(), operator[](Vec).
template <typename T, uint32_t N>
struct HostView {
    char* base;
    alpaka::Vec<uint32_t, N> ext;
    int64_t pitch[N];

    explicit HostView(OView const& v) : base(static_cast<char*>(v.data)) {
        for (uint32_t a = 0; a < N; ++a) {
            ext[a] = static_cast<uint32_t>(v.extents[a]);
            pitch[a] = v.pitches[a];
        }
    }
    alpaka::Vec<uint32_t, N> getExtents() const { return ext; }
    template <typename I>
    T& operator[](alpaka::Vec<I, N> const& idx) const {
        char* p = base;
        for (uint32_t a = 0; a < N; ++a) p += static_cast<int64_t>(idx[a]) * pitch[a];
        return *reinterpret_cast<T*>(p);
    }
};

struct HostAcc {};

template <typename T>
void scores(OView const* q, OView const* k, OView const* s, uint32_t g, int layout) {
    alpaka::nn::onAcc::internal::nn::AttentionScoresKernel<T> kernel{g, static_cast<alpaka::nn::AttentionKvLayout>(layout)};
    kernel(HostAcc{}, HostView<T, 4>(*s), HostView<T, 4>(*q), HostView<T, 4>(*k));
}

template <typename T>
void apply(OView const* p, OView const* v, OView const* o, uint32_t g, int layout) {
    alpaka::nn::onAcc::internal::nn::AttentionApplyKernel<T> kernel{g, static_cast<alpaka::nn::AttentionKvLayout>(layout)};
    kernel(HostAcc{}, HostView<T, 4>(*o), HostView<T, 4>(*p), HostView<T, 4>(*v));
}

template <typename T>
void embedding(OView const* ids, OView const* table, OView const* out) {
    alpaka::nn::onAcc::internal::nn::EmbeddingLookupKernel<T> kernel{};
    kernel(HostAcc{}, HostView<T, 2>(*out), HostView<uint32_t, 1>(*ids), HostView<T, 2>(*table));
}

template <typename T, uint32_t N>
void rms_norm_n(OView const* x, OView const* w, OView const* out, T eps) {
    alpaka::nn::onAcc::internal::nn::RmsNormKernel<T> kernel{eps};
    kernel(HostAcc{}, HostView<T, N>(*out), HostView<T, N>(*x), HostView<T, 1>(*w));
}

template <typename T>
int rms_norm(OView const* x, OView const* w, OView const* out, T eps) {
    switch (x->rank) {
        case 1: rms_norm_n<T, 1>(x, w, out, eps); return 0;
        case 2: rms_norm_n<T, 2>(x, w, out, eps); return 0;
        case 3: rms_norm_n<T, 3>(x, w, out, eps); return 0;
        case 4: rms_norm_n<T, 4>(x, w, out, eps); return 0;
        default: return 1;
    }
}

template <typename T>
void rope(OView const* in, OView const* cos_t, OView const* sin_t, OView const* out, int layout, uint32_t offset) {
    alpaka::nn::onAcc::internal::nn::RopeSingleKernel<T> kernel{offset, static_cast<alpaka::nn::RopeLayout>(layout)};
    kernel(HostAcc{}, HostView<T, 4>(*out), HostView<T, 4>(*in), HostView<T, 2>(*cos_t), HostView<T, 2>(*sin_t));
}

template <typename T, uint32_t N>
void softmax_n(OView const* in, OView const* out, uint32_t axis, bool causal, uint32_t qa, uint32_t ka) {
    alpaka::nn::onAcc::internal::nn::SoftmaxKernel<T> kernel{axis, causal, qa, ka};
    kernel(HostAcc{}, HostView<T, N>(*out), HostView<T, N>(*in));
}

template <typename T>
int softmax(OView const* in, OView const* out, uint32_t axis, int causal, uint32_t qa, uint32_t ka) {
    switch (in->rank) {
        case 1: softmax_n<T, 1>(in, out, axis, causal != 0, qa, ka); return 0;
        case 2: softmax_n<T, 2>(in, out, axis, causal != 0, qa, ka); return 0;
        case 3: softmax_n<T, 3>(in, out, axis, causal != 0, qa, ka); return 0;
        case 4: softmax_n<T, 4>(in, out, axis, causal != 0, qa, ka); return 0;
        default: return 1;
    }
}

template <typename T>
int masked_softmax(OView const* in, OView const* mask, OView const* out, uint32_t axis) {
    if (in->rank != 4) return 1;
    alpaka::nn::onAcc::internal::nn::MaskedSoftmaxKernel<T> kernel{axis};
    kernel(HostAcc{}, HostView<T, 4>(*out), HostView<T, 4>(*in), HostView<T, 4>(*mask));
    return 0;
}

}  // namespace


extern "C" {

void ref_attention_scores_f32(OView const* q, OView const* k, OView const* s, uint32_t g, int layout) {
    scores<float>(q, k, s, g, layout);
}
void ref_attention_scores_f64(OView const* q, OView const* k, OView const* s, uint32_t g, int layout) {
    scores<double>(q, k, s, g, layout);
}
void ref_attention_apply_f32(OView const* p, OView const* v, OView const* o, uint32_t g, int layout) {
    apply<float>(p, v, o, g, layout);
}
void ref_attention_apply_f64(OView const* p, OView const* v, OView const* o, uint32_t g, int layout) {
    apply<double>(p, v, o, g, layout);
}
void ref_embedding_lookup_f32(OView const* ids, OView const* table, OView const* out) {
    embedding<float>(ids, table, out);
}
void ref_embedding_lookup_f64(OView const* ids, OView const* table, OView const* out) {
    embedding<double>(ids, table, out);
}
int ref_rms_norm_f32(OView const* x, OView const* w, OView const* out, float eps) { return rms_norm<float>(x, w, out, eps); }
int ref_rms_norm_f64(OView const* x, OView const* w, OView const* out, double eps) {
    return rms_norm<double>(x, w, out, eps);
}
void ref_rope_f32(OView const* in, OView const* c, OView const* s, OView const* out, int layout, uint32_t offset) {
    rope<float>(in, c, s, out, layout, offset);
}
void ref_rope_f64(OView const* in, OView const* c, OView const* s, OView const* out, int layout, uint32_t offset) {
    rope<double>(in, c, s, out, layout, offset);
}
int ref_softmax_f32(OView const* in, OView const* out, uint32_t axis, int causal, uint32_t qa, uint32_t ka) {
    return softmax<float>(in, out, axis, causal, qa, ka);
}
int ref_softmax_f64(OView const* in, OView const* out, uint32_t axis, int causal, uint32_t qa, uint32_t ka) {
    return softmax<double>(in, out, axis, causal, qa, ka);
}
int ref_masked_softmax_f32(OView const* in, OView const* mask, OView const* out, uint32_t axis) {
    return masked_softmax<float>(in, mask, out, axis);
}
int ref_masked_softmax_f64(OView const* in, OView const* mask, OView const* out, uint32_t axis) {
    return masked_softmax<double>(in, mask, out, axis);
}

}  // extern "C"
