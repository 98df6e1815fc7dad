// mlp.cu -- linearBias, mlpForward and the gated mlp (reference:
// onHost/nn/mlp.hpp:33-338).
//
// The GEMMs run on cuBLAS (ann_gemm_*), as the reference's run on its vendor
// BLAS. What changes is the traffic around them:
//  - bias + activation is one pass over the GEMM output, in place
//    (ann_bias_add_* with an activation); the reference runs biasAdd into a
//    second buffer and then the activation in place;
//  - mlpForward feeds the caller's input to the first GEMM directly (the
//    reference copies it into scratch first) and ping-pongs the hidden
//    activations between two buffers instead of allocating two per layer;
//  - the gated mlp writes swiglu(gate, up) over gate, so it needs two
//    [batch, hidden] buffers, not three.
// Scratch is the caller's workspace when given, else a stream-ordered
// cudaMallocAsync / cudaFreeAsync on the call's stream (the counterpart of the
// reference's alloc + keepAlive(queue)).
#include "common.cuh"

namespace ann {
namespace {

template <typename T>
int gemm_t(ann_stream s, const ann_view* a, const ann_view* b, const ann_view* c) {
    if constexpr (sizeof(T) == 4) return ann_gemm_f32(s, a, b, c);
    else return ann_gemm_f64(s, a, b, c);
}

template <typename T>
int bias_t(ann_stream s, const ann_view* in, const ann_view* bias, int act, const ann_view* out) {
    if constexpr (sizeof(T) == 4) return ann_bias_add_f32(s, in, bias, act, out);
    else return ann_bias_add_f64(s, in, bias, act, out);
}

template <typename T>
int swiglu_t(ann_stream s, const ann_view* l, const ann_view* r, const ann_view* out) {
    if constexpr (sizeof(T) == 4) return ann_binary_f32(s, ANN_BINARY_SWIGLU, l, r, out, 0.0f);
    else return ann_binary_f64(s, ANN_BINARY_SWIGLU, l, r, out, 0.0);
}

ann_view dense2(void* p, int64_t rows, int64_t cols, size_t es) {
    ann_view v{};
    v.data = p;
    v.rank = 2;
    v.extents[0] = rows;
    v.extents[1] = cols;
    v.pitches[1] = static_cast<int64_t>(es);
    v.pitches[0] = cols * static_cast<int64_t>(es);
    return v;
}

// The caller's workspace, or a stream-ordered allocation freed (stream
// ordered) when the call returns.
struct Scratch {
    cudaStream_t stream;
    char* ptr = nullptr;
    bool owned = false;
    explicit Scratch(cudaStream_t s) : stream(s) {}
    Scratch(Scratch const&) = delete;
    Scratch& operator=(Scratch const&) = delete;
    int get(uint64_t need, void* workspace, uint64_t workspace_bytes, char const* what) {
        if (need == 0) return ANN_OK;
        if (workspace) {
            if (workspace_bytes < need)
                return fail(ANN_EINVAL, "%s: workspace of %llu bytes is below the %llu bytes needed.", what,
                            static_cast<unsigned long long>(workspace_bytes), static_cast<unsigned long long>(need));
            ptr = static_cast<char*>(workspace);
            return ANN_OK;
        }
        void* p = nullptr;
        cudaError_t const e = cudaMallocAsync(&p, need, stream);
        if (e != cudaSuccess) return fail(ANN_ECUDA, "%s: cudaMallocAsync: %s", what, cudaGetErrorString(e));
        ptr = static_cast<char*>(p);
        owned = true;
        return ANN_OK;
    }
    ~Scratch() {
        if (owned) cudaFreeAsync(ptr, stream);
    }
};

// Shape checks of mlpForward (mlp.hpp:171-193). On success *batch, *max_hidden
// (largest out extent of the layers before the last) and *scratch_elems.
int mlp_forward_shapes(const ann_view* input, int32_t n_layers, const ann_view* weights, const ann_view* biases,
                       const ann_view* output, size_t es, int64_t* batch, int64_t* max_hidden,
                       int64_t* scratch_elems) {
    if (n_layers <= 0 || !weights || !biases) return fail(ANN_EINVAL, "mlpForward: at least one layer is required.");
    Dims in, out;
    ANN_TRY(to_dims(input, es, "mlpForward input", in));
    if (in.rank != 2) return fail(ANN_EINVAL, "mlpForward expects a [batch, in] input.");
    int64_t expected = in.ext[1];
    int64_t hidden = 0;
    for (int32_t l = 0; l < n_layers; ++l) {
        Dims w, b;
        ANN_TRY(to_dims(&weights[l], es, "mlpForward weight", w));
        ANN_TRY(to_dims(&biases[l], es, "mlpForward bias", b));
        if (w.rank != 2) return fail(ANN_EINVAL, "mlpForward: layer %d weight is not [in, out].", l);
        if (w.ext[0] != expected)
            return fail(ANN_EINVAL, "mlpForward: layer %d weight expects in=%lld but previous out=%lld.", l,
                        static_cast<long long>(w.ext[0]), static_cast<long long>(expected));
        if (b.ext[0] != w.ext[1])
            return fail(ANN_EINVAL, "mlpForward: layer %d bias extent does not match the weight out extent.", l);
        expected = w.ext[1];
        if (l + 1 < n_layers && w.ext[1] > hidden) hidden = w.ext[1];
    }
    ANN_TRY(to_dims(output, es, "mlpForward output", out));
    if (out.rank != 2 || out.ext[0] != in.ext[0] || out.ext[1] != expected)
        return fail(ANN_EINVAL, "mlpForward: output extent does not match batch x last-out.");
    *batch = in.ext[0];
    *max_hidden = hidden;
    *scratch_elems = static_cast<int64_t>(n_layers >= 3 ? 2 : n_layers - 1) * in.ext[0] * hidden;
    return ANN_OK;
}

template <typename T>
int mlp_forward(ann_stream stream, const ann_view* input, int32_t n_layers, const ann_view* weights,
                const ann_view* biases, int32_t hidden_act, int32_t last_act, const ann_view* output,
                void* workspace, uint64_t workspace_bytes) {
    int64_t batch = 0, hidden = 0, elems = 0;
    ANN_TRY(mlp_forward_shapes(input, n_layers, weights, biases, output, sizeof(T), &batch, &hidden, &elems));
    if (hidden_act < ANN_ACT_NONE || hidden_act > ANN_ACT_GELU || last_act < ANN_ACT_NONE || last_act > ANN_ACT_GELU)
        return fail(ANN_EINVAL, "mlpForward: unsupported activation.");
    if (batch == 0) return ANN_OK;
    Scratch scratch(as_stream(stream));
    ANN_TRY(scratch.get(static_cast<uint64_t>(elems) * sizeof(T), workspace, workspace_bytes, "mlpForward"));
    ann_view prev = *input;
    for (int32_t l = 0; l < n_layers; ++l) {
        int64_t const out_ext = weights[l].extents[1];
        if (l + 1 == n_layers) {
            ANN_TRY(gemm_t<T>(stream, &prev, &weights[l], output));
            ANN_TRY(bias_t<T>(stream, output, &biases[l], last_act, output));
        } else {
            ann_view const next = dense2(scratch.ptr + (l % 2) * batch * hidden * sizeof(T), batch, out_ext, sizeof(T));
            ANN_TRY(gemm_t<T>(stream, &prev, &weights[l], &next));
            ANN_TRY(bias_t<T>(stream, &next, &biases[l], hidden_act, &next));
            prev = next;
        }
    }
    return ANN_OK;
}

// mlp (mlp.hpp:307-337): output = swiglu(input.Wgate, input.Wup) . Wdown.
template <typename T>
int gated_mlp(ann_stream stream, const ann_view* input, const ann_view* wgate, const ann_view* wup,
              const ann_view* wdown, const ann_view* output, void* workspace, uint64_t workspace_bytes) {
    Dims in, g, u;
    ANN_TRY(to_dims(input, sizeof(T), "mlp input", in));
    ANN_TRY(to_dims(wgate, sizeof(T), "mlp Wgate", g));
    ANN_TRY(to_dims(wup, sizeof(T), "mlp Wup", u));
    if (in.rank != 2 || g.rank != 2 || u.rank != 2) return fail(ANN_EINVAL, "gemm expects rank-2 operands.");
    if (g.ext[1] != u.ext[1]) return fail(ANN_EINVAL, "binaryOp shape mismatch.");  // swiglu(gate, up)
    Dims d, o;
    ANN_TRY(to_dims(wdown, sizeof(T), "mlp Wdown", d));
    ANN_TRY(to_dims(output, sizeof(T), "mlp output", o));
    // The three GEMMs' shapes, before any of them is enqueued.
    if (d.rank != 2 || o.rank != 2) return fail(ANN_EINVAL, "gemm expects rank-2 operands.");
    if (g.ext[0] != in.ext[1] || u.ext[0] != in.ext[1] || d.ext[0] != g.ext[1] || o.ext[0] != in.ext[0] ||
        o.ext[1] != d.ext[1])
        return fail(ANN_EINVAL, "gemm shape mismatch.");
    int64_t const batch = in.ext[0], hidden = g.ext[1];
    if (batch == 0) return gemm_t<T>(stream, input, wdown, output);  // validates, computes nothing
    Scratch scratch(as_stream(stream));
    ANN_TRY(scratch.get(static_cast<uint64_t>(2 * batch * hidden) * sizeof(T), workspace, workspace_bytes, "mlp"));
    ann_view const gate = dense2(scratch.ptr, batch, hidden, sizeof(T));
    ann_view const up = dense2(scratch.ptr + batch * hidden * sizeof(T), batch, hidden, sizeof(T));
    ANN_TRY(gemm_t<T>(stream, input, wgate, &gate));
    ANN_TRY(gemm_t<T>(stream, input, wup, &up));
    ANN_TRY(swiglu_t<T>(stream, &gate, &up, &gate));
    return gemm_t<T>(stream, &gate, wdown, output);
}

}  // namespace
}  // namespace ann

extern "C" {

int ann_linear_bias_f32(ann_stream s, const ann_view* input, const ann_view* weight, const ann_view* bias,
                        int32_t act, const ann_view* output) {
    ANN_API_BEGIN
    ANN_TRY(ann_gemm_f32(s, input, weight, output));
    return ann_bias_add_f32(s, output, bias, act, output);
    ANN_API_END
}
int ann_linear_bias_f64(ann_stream s, const ann_view* input, const ann_view* weight, const ann_view* bias,
                        int32_t act, const ann_view* output) {
    ANN_API_BEGIN
    ANN_TRY(ann_gemm_f64(s, input, weight, output));
    return ann_bias_add_f64(s, output, bias, act, output);
    ANN_API_END
}

int ann_mlp_forward_workspace_bytes(const ann_view* input, int32_t n_layers, const ann_view* weights,
                                    const ann_view* biases, const ann_view* output, size_t element_size,
                                    uint64_t* bytes) {
    ANN_API_BEGIN
    if (!bytes) return ann::fail(ANN_EINVAL, "mlpForward: bytes is NULL.");
    if (element_size != 4 && element_size != 8) return ann::fail(ANN_EINVAL, "mlpForward: element size 4 or 8.");
    int64_t batch = 0, hidden = 0, elems = 0;
    ANN_TRY(ann::mlp_forward_shapes(input, n_layers, weights, biases, output, element_size, &batch, &hidden, &elems));
    *bytes = static_cast<uint64_t>(elems) * element_size;
    return ANN_OK;
    ANN_API_END
}

int ann_mlp_forward_f32(ann_stream s, const ann_view* input, int32_t n_layers, const ann_view* weights,
                        const ann_view* biases, int32_t hidden_act, int32_t last_act, const ann_view* output,
                        void* workspace, uint64_t workspace_bytes) {
    ANN_API_BEGIN
    return ann::mlp_forward<float>(s, input, n_layers, weights, biases, hidden_act, last_act, output, workspace,
                                   workspace_bytes);
    ANN_API_END
}
int ann_mlp_forward_f64(ann_stream s, const ann_view* input, int32_t n_layers, const ann_view* weights,
                        const ann_view* biases, int32_t hidden_act, int32_t last_act, const ann_view* output,
                        void* workspace, uint64_t workspace_bytes) {
    ANN_API_BEGIN
    return ann::mlp_forward<double>(s, input, n_layers, weights, biases, hidden_act, last_act, output, workspace,
                                    workspace_bytes);
    ANN_API_END
}

int ann_mlp_f32(ann_stream s, const ann_view* input, const ann_view* wgate, const ann_view* wup,
                const ann_view* wdown, const ann_view* output, void* workspace, uint64_t workspace_bytes) {
    ANN_API_BEGIN
    return ann::gated_mlp<float>(s, input, wgate, wup, wdown, output, workspace, workspace_bytes);
    ANN_API_END
}
int ann_mlp_f64(ann_stream s, const ann_view* input, const ann_view* wgate, const ann_view* wup,
                const ann_view* wdown, const ann_view* output, void* workspace, uint64_t workspace_bytes) {
    ANN_API_BEGIN
    return ann::gated_mlp<double>(s, input, wgate, wup, wdown, output, workspace, workspace_bytes);
    ANN_API_END
}

}  // extern "C"
