/*
 * alpakann_b200/onHost.hpp -- C++20 drop-in for alpakaNN's attention path.
 *
 * Same namespaces, function names, template parameter (T_Type), argument
 * order, defaults and exceptions as the reference's header-only host API
 * (include/alpaka/nn/onHost/nn/{embedding,rms_norm,attention,rope,softmax}.hpp,
 * include/alpaka/nn/onHost/ops/elementwise.hpp, include/alpaka/nn/onHost/matrix/gemm.hpp),
 * implemented on the sm_100a kernels behind include/ann_b200.h.
 *
 *  - queue: anything nativeStream() understands -- alpaka::nn::b200::Queue
 *    (one CUDA stream), a cudaStream_t, or a type with getNativeHandle().
 *  - exec: accepted and ignored (it selected alpaka's thread mapping).
 *  - views: any type with data(), getExtents() and getPitches() (BYTE
 *    pitches, alpaka's convention), e.g. alpaka::nn::b200::View.
 *  - ANN_EINVAL becomes std::invalid_argument with the reference's message,
 *    every other failure std::runtime_error.
 */
#pragma once

#include <cuda_runtime.h>

#include <array>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <span>
#include <sstream>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

#include "../ann_b200.h"

namespace alpaka::nn {
// nn/attention.hpp:10-14 and nn/rope.hpp:10-14
enum class AttentionKvLayout { BTHD = ANN_LAYOUT_BTHD, BHTD = ANN_LAYOUT_BHTD };
enum class RopeLayout { BTHD = ANN_LAYOUT_BTHD, BHTD = ANN_LAYOUT_BHTD };
}  // namespace alpaka::nn

namespace alpaka::nn::b200 {

// In-order queue = one CUDA stream on one device.
struct Queue {
    cudaStream_t stream = nullptr;
    int device = 0;
    bool owned = false;

    Queue() = default;
    explicit Queue(int dev) : device(dev), owned(true) {
        cudaSetDevice(dev);
        if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess)
            throw std::runtime_error("alpakann_b200: cudaStreamCreate failed");
    }
    Queue(cudaStream_t s, int dev) : stream(s), device(dev) {}
    Queue(Queue const&) = delete;
    Queue& operator=(Queue const&) = delete;
    ~Queue() {
        if (owned && stream) cudaStreamDestroy(stream);
    }
    void wait() const {
        if (cudaStreamSynchronize(stream) != cudaSuccess) throw std::runtime_error("alpakann_b200: stream error");
    }
    cudaStream_t getNativeHandle() const { return stream; }
};

// Strided view over device (or host) memory: extents and BYTE pitches.
template <typename T, std::size_t R>
struct View {
    using value_type = T;
    T* ptr = nullptr;
    std::array<int64_t, R> extents{};
    std::array<int64_t, R> pitches{};
    T* data() const { return ptr; }
    std::array<int64_t, R> const& getExtents() const { return extents; }
    std::array<int64_t, R> const& getPitches() const { return pitches; }
};

// Dense row-major view (alpaka::makeView analogue).
template <typename T, std::size_t R>
View<T, R> makeView(T* ptr, std::array<int64_t, R> const& ext) {
    View<T, R> v;
    v.ptr = ptr;
    v.extents = ext;
    int64_t p = sizeof(T);
    for (std::size_t i = R; i-- > 0;) {
        v.pitches[i] = p;
        p *= ext[i];
    }
    return v;
}

// Sub-view at an element offset (getSubView analogue, same pitches).
template <typename T, std::size_t R>
View<T, R> subView(View<T, R> const& src, std::array<int64_t, R> const& offset, std::array<int64_t, R> const& ext) {
    View<T, R> v = src;
    char* p = reinterpret_cast<char*>(src.ptr);
    for (std::size_t i = 0; i < R; ++i) p += offset[i] * src.pitches[i];
    v.ptr = reinterpret_cast<T*>(p);
    v.extents = ext;
    return v;
}

// Owning one-dimensional device allocation: what alpaka::onHost::alloc<T>(
// device, Vec{n}) returns to loadBinaryTensor's caller. Allocated on the
// current device; freed (cudaFree) when it goes out of scope.
template <typename T>
class DeviceBuffer {
public:
    using value_type = T;
    DeviceBuffer() = default;
    explicit DeviceBuffer(int64_t n) : extents_{n}, pitches_{static_cast<int64_t>(sizeof(T))} {
        if (n > 0 && cudaMalloc(reinterpret_cast<void**>(&ptr_), static_cast<std::size_t>(n) * sizeof(T)) != cudaSuccess) {
            ptr_ = nullptr;
            throw std::runtime_error("alpakann_b200: cudaMalloc failed");
        }
    }
    DeviceBuffer(DeviceBuffer&& o) noexcept : ptr_(std::exchange(o.ptr_, nullptr)), extents_(o.extents_), pitches_(o.pitches_) {}
    DeviceBuffer& operator=(DeviceBuffer&& o) noexcept {
        if (this != &o) {
            reset();
            ptr_ = std::exchange(o.ptr_, nullptr);
            extents_ = o.extents_;
            pitches_ = o.pitches_;
        }
        return *this;
    }
    DeviceBuffer(DeviceBuffer const&) = delete;
    DeviceBuffer& operator=(DeviceBuffer const&) = delete;
    ~DeviceBuffer() { reset(); }
    T* data() const { return ptr_; }
    std::array<int64_t, 1> const& getExtents() const { return extents_; }
    std::array<int64_t, 1> const& getPitches() const { return pitches_; }

private:
    void reset() {
        if (ptr_) cudaFree(ptr_);
        ptr_ = nullptr;
    }
    T* ptr_ = nullptr;
    std::array<int64_t, 1> extents_{};
    std::array<int64_t, 1> pitches_{};
};

namespace detail {
template <typename E>
constexpr std::size_t rank_of(E const& e) {
    if constexpr (requires { e.size(); })
        return static_cast<std::size_t>(e.size());
    else
        return static_cast<std::size_t>(std::remove_cvref_t<E>::dim());
}

template <typename V>
ann_view to_ann(V const& v) {
    ann_view a{};
    auto const& ext = v.getExtents();
    auto const& pit = v.getPitches();
    std::size_t const r = rank_of(ext);
    if (r > ANN_MAX_RANK) throw std::invalid_argument("alpakann_b200: view rank exceeds 8.");
    a.data = const_cast<void*>(static_cast<void const*>(v.data()));
    a.rank = static_cast<int32_t>(r);
    for (std::size_t i = 0; i < r; ++i) {
        a.extents[i] = static_cast<int64_t>(ext[i]);
        a.pitches[i] = static_cast<int64_t>(pit[i]);
    }
    return a;
}

template <typename Q>
ann_stream stream_of(Q& q) {
    if constexpr (std::is_same_v<std::remove_cvref_t<Q>, cudaStream_t>)
        return reinterpret_cast<ann_stream>(q);
    else
        return reinterpret_cast<ann_stream>(q.getNativeHandle());
}

inline void check(int rc) {
    if (rc == ANN_OK) return;
    std::string msg = ann_last_error();
    if (rc == ANN_EINVAL) throw std::invalid_argument(msg);
    throw std::runtime_error("alpakann_b200: " + msg);
}

template <typename T>
constexpr bool is_f32 = std::is_same_v<T, float>;
template <typename T>
constexpr bool is_f64 = std::is_same_v<T, double>;
template <typename T>
constexpr void require_float() {
    static_assert(is_f32<T> || is_f64<T>, "alpakann_b200 supports float and double");
}

// Element type of a view (its data() pointee) and its ANN_DTYPE_* code.
template <typename V>
using elem_of = std::remove_cv_t<std::remove_pointer_t<decltype(std::declval<V const&>().data())>>;
template <typename E>
constexpr int32_t dtype_code() {
    if constexpr (std::is_same_v<E, float>) return ANN_DTYPE_F32;
    else if constexpr (std::is_same_v<E, double>) return ANN_DTYPE_F64;
    else if constexpr (std::is_same_v<E, int32_t>) return ANN_DTYPE_I32;
    else if constexpr (std::is_same_v<E, uint32_t>) return ANN_DTYPE_U32;
    else {
        static_assert(std::is_same_v<E, int64_t>, "alpakann_b200: float, double, int32, uint32 or int64 elements");
        return ANN_DTYPE_I64;
    }
}

template <typename T, typename Q>
void unary(Q& queue, int32_t op, ann_view const& i, ann_view const& o, T scalar = T(0)) {
    require_float<T>();
    if constexpr (is_f32<T>)
        check(ann_unary_f32(stream_of(queue), op, &i, &o, scalar));
    else
        check(ann_unary_f64(stream_of(queue), op, &i, &o, scalar));
}
template <typename T, typename Q>
void binary(Q& queue, int32_t op, ann_view const& l, ann_view const& r, ann_view const& o, T alpha = T(0)) {
    require_float<T>();
    if constexpr (is_f32<T>)
        check(ann_binary_f32(stream_of(queue), op, &l, &r, &o, alpha));
    else
        check(ann_binary_f64(stream_of(queue), op, &l, &r, &o, alpha));
}
template <typename T, typename Q>
void reduce(Q& queue, int32_t op, ann_view const& i, ann_view const& o, uint32_t axis) {
    require_float<T>();
    if constexpr (is_f32<T>)
        check(ann_reduce_f32(stream_of(queue), op, &i, &o, axis));
    else
        check(ann_reduce_f64(stream_of(queue), op, &i, &o, axis));
}

// ALPAKANN_DEBUG_ATTENTION_TRACE (onHost/nn/attention.hpp:24-34)
inline bool attention_trace_enabled() {
    auto const* env = std::getenv("ALPAKANN_DEBUG_ATTENTION_TRACE");
    return env != nullptr && env[0] != '\0' && env[0] != '0';
}
inline std::string ext_str(ann_view const& v) {
    std::ostringstream os;
    os << "{";
    for (int i = 0; i < v.rank; ++i) os << (i ? ", " : "") << v.extents[i];
    os << "}";
    return os.str();
}
}  // namespace detail
}  // namespace alpaka::nn::b200

namespace alpaka::nn::onHost {

// onHost/matrix/gemm.hpp:28-33 -- C = A * B on cuBLAS
template <typename T_Type = float>
void gemm(auto& queue, auto const& A, auto const& B, auto& C) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto a = d::to_ann(A), b = d::to_ann(B), c = d::to_ann(C);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_gemm_f32(d::stream_of(queue), &a, &b, &c));
    else
        d::check(ann_gemm_f64(d::stream_of(queue), &a, &b, &c));
}

}  // namespace alpaka::nn::onHost

namespace alpaka::nn::onHost {
// onHost/core/binary.hpp:33-39
struct TensorSpec {
    std::string name;
    std::size_t offsetBytes;
    std::size_t count;
    std::vector<std::size_t> shape;
};

namespace detail {
inline ann_tensor_spec to_ann(TensorSpec const& spec, std::vector<uint64_t>& shape) {
    shape.assign(spec.shape.begin(), spec.shape.end());
    ann_tensor_spec s{};
    s.name = spec.name.c_str();
    s.offset_bytes = spec.offsetBytes;
    s.count = spec.count;
    s.shape = shape.empty() ? nullptr : shape.data();
    s.shape_rank = static_cast<int32_t>(shape.size());
    return s;
}
}  // namespace detail

// sha256File (onHost/core/binary.hpp:212-232): 64 lowercase hex digits;
// std::runtime_error if the file cannot be opened or read.
inline std::string sha256File(std::string const& path) {
    char hex[65] = {};
    b200::detail::check(ann_sha256_file(path.c_str(), hex));
    return std::string(hex);
}

// loadBinaryTensor<T> (onHost/core/binary.hpp:234-323): the tensor's count
// elements in a new device buffer on the current device, copied on `queue`.
// std::invalid_argument for a bad layout, std::runtime_error for file errors
// and a digest mismatch, all raised before the buffer is allocated.
template <typename T_Type>
auto loadBinaryTensor(auto& queue, std::string const& path, TensorSpec const& spec,
                      std::string const& expectedSha256 = std::string{}) {
    static_assert(std::is_same_v<T_Type, float> || std::is_same_v<T_Type, double>,
                  "alpaka::nn::onHost::loadBinaryTensor supports only float32 and float64 tensors.");
    std::vector<uint64_t> shape;
    ann_tensor_spec const s = detail::to_ann(spec, shape);
    // Every check (and the digest) with nothing allocated yet, then the load.
    b200::detail::check(ann_load_binary_tensor(b200::detail::stream_of(queue), path.c_str(), &s, sizeof(T_Type),
                                               expectedSha256.c_str(), nullptr));
    b200::DeviceBuffer<T_Type> buffer(static_cast<int64_t>(spec.count));
    b200::detail::check(
        ann_load_binary_tensor(b200::detail::stream_of(queue), path.c_str(), &s, sizeof(T_Type), "", buffer.data()));
    return buffer;
}
}  // namespace alpaka::nn::onHost

namespace alpaka::nn::onHost::ops {

// onHost/ops/elementwise.hpp:330-334
template <typename T_Type>
void scale(auto& queue, auto /*exec*/, auto const& in, T_Type scalar, auto& out) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto i = d::to_ann(in), o = d::to_ann(out);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_scale_f32(d::stream_of(queue), &i, scalar, &o));
    else
        d::check(ann_scale_f64(d::stream_of(queue), &i, scalar, &o));
}

// onHost/ops/elementwise.hpp:250-254: every element of out = value, in out's element type.
template <typename T_Value>
void fill(auto& queue, auto /*exec*/, auto& out, T_Value value) {
    namespace d = alpaka::nn::b200::detail;
    using E = d::elem_of<std::remove_cvref_t<decltype(out)>>;
    E const v = static_cast<E>(value);
    auto o = d::to_ann(out);
    d::check(ann_fill(d::stream_of(queue), &o, d::dtype_code<E>(), &v));
}

// :256-268
void copy(auto& queue, auto /*exec*/, auto const& in, auto& out) {
    namespace d = alpaka::nn::b200::detail;
    using E = d::elem_of<std::remove_cvref_t<decltype(out)>>;
    d::unary<E>(queue, ANN_UNARY_COPY, d::to_ann(in), d::to_ann(out));
}

// :306-337
template <typename T_Type>
void add(auto& queue, auto /*exec*/, auto const& lhs, auto const& rhs, auto& out) {
    namespace d = alpaka::nn::b200::detail;
    d::binary<T_Type>(queue, ANN_BINARY_ADD, d::to_ann(lhs), d::to_ann(rhs), d::to_ann(out));
}
template <typename T_Type>
void sub(auto& queue, auto /*exec*/, auto const& lhs, auto const& rhs, auto& out) {
    namespace d = alpaka::nn::b200::detail;
    d::binary<T_Type>(queue, ANN_BINARY_SUB, d::to_ann(lhs), d::to_ann(rhs), d::to_ann(out));
}
template <typename T_Type>
void mul(auto& queue, auto /*exec*/, auto const& lhs, auto const& rhs, auto& out) {
    namespace d = alpaka::nn::b200::detail;
    d::binary<T_Type>(queue, ANN_BINARY_MUL, d::to_ann(lhs), d::to_ann(rhs), d::to_ann(out));
}
template <typename T_Type>
void div(auto& queue, auto /*exec*/, auto const& lhs, auto const& rhs, auto& out) {
    namespace d = alpaka::nn::b200::detail;
    d::binary<T_Type>(queue, ANN_BINARY_DIV, d::to_ann(lhs), d::to_ann(rhs), d::to_ann(out));
}
template <typename T_Type>
void axpy(auto& queue, auto /*exec*/, T_Type alpha, auto const& x, auto const& y, auto& out) {
    namespace d = alpaka::nn::b200::detail;
    d::binary<T_Type>(queue, ANN_BINARY_AXPY, d::to_ann(x), d::to_ann(y), d::to_ann(out), alpha);
}

// :338-353
void biasAdd(auto& queue, auto /*exec*/, auto const& input, auto const& bias, auto& out) {
    namespace d = alpaka::nn::b200::detail;
    using E = d::elem_of<std::remove_cvref_t<decltype(out)>>;
    d::require_float<E>();
    auto i = d::to_ann(input), b = d::to_ann(bias), o = d::to_ann(out);
    if constexpr (d::is_f32<E>)
        d::check(ann_bias_add_f32(d::stream_of(queue), &i, &b, ANN_ACT_NONE, &o));
    else
        d::check(ann_bias_add_f64(d::stream_of(queue), &i, &b, ANN_ACT_NONE, &o));
}

// :355-361
template <typename T_Out>
void cast(auto& queue, auto /*exec*/, auto const& in, auto& out) {
    namespace d = alpaka::nn::b200::detail;
    using In = d::elem_of<std::remove_cvref_t<decltype(in)>>;
    static_assert(std::is_same_v<T_Out, d::elem_of<std::remove_cvref_t<decltype(out)>>>,
                  "cast<T_Out>: out must hold T_Out elements");
    auto i = d::to_ann(in), o = d::to_ann(out);
    d::check(ann_cast(d::stream_of(queue), &i, d::dtype_code<In>(), &o, d::dtype_code<T_Out>()));
}

// :363-414, the transcendental and activation operators
#define ANN_B200_UNARY(name, code)                                                     \
    template <typename T_Type>                                                         \
    void name(auto& queue, auto /*exec*/, auto const& in, auto& out) {                 \
        namespace d = alpaka::nn::b200::detail;                                        \
        d::unary<T_Type>(queue, code, d::to_ann(in), d::to_ann(out));                  \
    }
ANN_B200_UNARY(exp, ANN_UNARY_EXP)
ANN_B200_UNARY(sqrt, ANN_UNARY_SQRT)
ANN_B200_UNARY(rsqrt, ANN_UNARY_RSQRT)
ANN_B200_UNARY(relu, ANN_UNARY_RELU)
ANN_B200_UNARY(sigmoid, ANN_UNARY_SIGMOID)
ANN_B200_UNARY(silu, ANN_UNARY_SILU)
ANN_B200_UNARY(gelu, ANN_UNARY_GELU)
#undef ANN_B200_UNARY

template <typename T_Type>
void swiglu(auto& queue, auto /*exec*/, auto const& lhs, auto const& rhs, auto& out) {
    namespace d = alpaka::nn::b200::detail;
    d::binary<T_Type>(queue, ANN_BINARY_SWIGLU, d::to_ann(lhs), d::to_ann(rhs), d::to_ann(out));
}

// onHost/ops/reduction.hpp:190-289
template <typename T_Type>
void reduceSum(auto& queue, auto /*exec*/, auto const& in, auto& out, uint32_t axis) {
    namespace d = alpaka::nn::b200::detail;
    d::reduce<T_Type>(queue, ANN_REDUCE_SUM, d::to_ann(in), d::to_ann(out), axis);
}
template <typename T_Type>
void reduceMax(auto& queue, auto /*exec*/, auto const& in, auto& out, uint32_t axis) {
    namespace d = alpaka::nn::b200::detail;
    d::reduce<T_Type>(queue, ANN_REDUCE_MAX, d::to_ann(in), d::to_ann(out), axis);
}
template <typename T_Type>
void reduceMean(auto& queue, auto /*exec*/, auto const& in, auto& out, uint32_t axis) {
    namespace d = alpaka::nn::b200::detail;
    d::reduce<T_Type>(queue, ANN_REDUCE_MEAN, d::to_ann(in), d::to_ann(out), axis);
}
template <typename T_Type>
void reduceSumSquares(auto& queue, auto /*exec*/, auto const& in, auto& out, uint32_t axis) {
    namespace d = alpaka::nn::b200::detail;
    d::reduce<T_Type>(queue, ANN_REDUCE_SUM_SQUARES, d::to_ann(in), d::to_ann(out), axis);
}
template <typename T_Type>
void dot(auto& queue, auto /*exec*/, auto const& lhs, auto const& rhs, auto& out, uint32_t axis) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto l = d::to_ann(lhs), r = d::to_ann(rhs), o = d::to_ann(out);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_dot_f32(d::stream_of(queue), &l, &r, &o, axis));
    else
        d::check(ann_dot_f64(d::stream_of(queue), &l, &r, &o, axis));
}
// reduction.hpp:285-288
inline auto makeReducedExtents(auto extents, uint32_t axis) {
    extents[axis] = 1;
    return extents;
}

}  // namespace alpaka::nn::onHost::ops

namespace alpaka::nn::onHost::nn {

// onHost/nn/embedding.hpp:17-36
template <typename T_Type>
void embeddingLookup(auto& queue, auto /*exec*/, auto const& tokenIds, auto const& embedding, auto& output) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto ids = d::to_ann(tokenIds), e = d::to_ann(embedding), o = d::to_ann(output);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_embedding_lookup_f32(d::stream_of(queue), &ids, &e, &o));
    else
        d::check(ann_embedding_lookup_f64(d::stream_of(queue), &ids, &e, &o));
}

// onHost/nn/rms_norm.hpp:17-35
template <typename T_Type>
void rmsNorm(auto& queue, auto /*exec*/, auto const& input, auto const& weight, auto& output, T_Type epsilon) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto i = d::to_ann(input), w = d::to_ann(weight), o = d::to_ann(output);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_rms_norm_f32(d::stream_of(queue), &i, &w, &o, epsilon));
    else
        d::check(ann_rms_norm_f64(d::stream_of(queue), &i, &w, &o, epsilon));
}

// outputProjection (onHost/nn/attention.hpp:112-116) then ops::add of the
// residual, fused: output = residual + input . Wo (residual may be output).
template <typename T_Type>
void outputProjectionResidual(auto& queue, auto const& input, auto const& Wo, auto const& residual, auto& output) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto i = d::to_ann(input), w = d::to_ann(Wo), r = d::to_ann(residual), o = d::to_ann(output);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_output_projection_residual_f32(d::stream_of(queue), &i, &w, &r, &o));
    else
        d::check(ann_output_projection_residual_f64(d::stream_of(queue), &i, &w, &r, &o));
}

// New K/V rows (BTHD) into BHTD caches at tokens [position, position + Tn); with
// RoPE tables K is rotated on the way, as ropeInPlace does.
template <typename T_Type>
void kvCacheAppend(auto& queue, auto /*exec*/, auto const& kNew, auto const& vNew, auto& kCache, auto& vCache,
                   uint32_t position) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto kn = d::to_ann(kNew), vn = d::to_ann(vNew), kc = d::to_ann(kCache), vc = d::to_ann(vCache);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_kv_cache_append_f32(d::stream_of(queue), &kn, &vn, &kc, &vc, nullptr, nullptr, position));
    else
        d::check(ann_kv_cache_append_f64(d::stream_of(queue), &kn, &vn, &kc, &vc, nullptr, nullptr, position));
}
template <typename T_Type>
void kvCacheAppend(auto& queue, auto /*exec*/, auto const& kNew, auto const& vNew, auto& kCache, auto& vCache,
                   auto const& cosTable, auto const& sinTable, uint32_t position) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto kn = d::to_ann(kNew), vn = d::to_ann(vNew), kc = d::to_ann(kCache), vc = d::to_ann(vCache);
    auto c = d::to_ann(cosTable), s = d::to_ann(sinTable);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_kv_cache_append_f32(d::stream_of(queue), &kn, &vn, &kc, &vc, &c, &s, position));
    else
        d::check(ann_kv_cache_append_f64(d::stream_of(queue), &kn, &vn, &kc, &vc, &c, &s, position));
}

// embeddingLookup (onHost/nn/embedding.hpp:17-36) then rmsNorm
// (onHost/nn/rms_norm.hpp:17-35) in one launch, bit for bit their result.
template <typename T_Type>
void embeddingRmsNorm(auto& queue, auto /*exec*/, auto const& tokenIds, auto const& embedding, auto const& weight,
                      auto& output, T_Type epsilon) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto t = d::to_ann(tokenIds), e = d::to_ann(embedding), w = d::to_ann(weight), o = d::to_ann(output);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_embedding_rms_norm_f32(d::stream_of(queue), &t, &e, &w, &o, epsilon));
    else
        d::check(ann_embedding_rms_norm_f64(d::stream_of(queue), &t, &e, &w, &o, epsilon));
}

// onHost/nn/attention.hpp:38-52
template <typename T_Type>
void qkvProjection(auto& queue, auto const& input, auto const& Wq, auto const& Wk, auto const& Wv, auto& Q, auto& K,
                   auto& V) {
    alpaka::nn::onHost::gemm<T_Type>(queue, input, Wq, Q);
    alpaka::nn::onHost::gemm<T_Type>(queue, input, Wk, K);
    alpaka::nn::onHost::gemm<T_Type>(queue, input, Wv, V);
}

// onHost/nn/attention.hpp:112-116
template <typename T_Type>
void outputProjection(auto& queue, auto const& input, auto const& Wo, auto& output) {
    alpaka::nn::onHost::gemm<T_Type>(queue, input, Wo, output);
}

// onHost/nn/attention.hpp:54-81
template <typename T_Type>
void attentionScores(auto& queue, auto /*exec*/, auto const& Q, auto const& K, auto& scores,
                     uint32_t queriesPerKvGroup = 1u,
                     alpaka::nn::AttentionKvLayout kvLayout = alpaka::nn::AttentionKvLayout::BTHD) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    if (queriesPerKvGroup == 0u) throw std::invalid_argument{"attentionScores requires queriesPerKvGroup > 0."};
    auto q = d::to_ann(Q), k = d::to_ann(K), s = d::to_ann(scores);
    if (d::attention_trace_enabled())
        std::fprintf(stderr, "attentionScores q=%s k=%s scores=%s queriesPerKvGroup=%u layout=%s\n",
                     d::ext_str(q).c_str(), d::ext_str(k).c_str(), d::ext_str(s).c_str(), queriesPerKvGroup,
                     kvLayout == alpaka::nn::AttentionKvLayout::BTHD ? "BTHD" : "BHTD");
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_attention_scores_f32(d::stream_of(queue), &q, &k, &s, queriesPerKvGroup,
                                          static_cast<int32_t>(kvLayout)));
    else
        d::check(ann_attention_scores_f64(d::stream_of(queue), &q, &k, &s, queriesPerKvGroup,
                                          static_cast<int32_t>(kvLayout)));
}

// onHost/nn/attention.hpp:83-110
template <typename T_Type>
void attentionApply(auto& queue, auto /*exec*/, auto const& probs, auto const& values, auto& out,
                    uint32_t queriesPerKvGroup = 1u,
                    alpaka::nn::AttentionKvLayout kvLayout = alpaka::nn::AttentionKvLayout::BTHD) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    if (queriesPerKvGroup == 0u) throw std::invalid_argument{"attentionApply requires queriesPerKvGroup > 0."};
    auto p = d::to_ann(probs), v = d::to_ann(values), o = d::to_ann(out);
    if (d::attention_trace_enabled())
        std::fprintf(stderr, "attentionApply probs=%s values=%s out=%s queriesPerKvGroup=%u layout=%s\n",
                     d::ext_str(p).c_str(), d::ext_str(v).c_str(), d::ext_str(o).c_str(), queriesPerKvGroup,
                     kvLayout == alpaka::nn::AttentionKvLayout::BTHD ? "BTHD" : "BHTD");
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_attention_apply_f32(d::stream_of(queue), &p, &v, &o, queriesPerKvGroup,
                                         static_cast<int32_t>(kvLayout)));
    else
        d::check(ann_attention_apply_f64(d::stream_of(queue), &p, &v, &o, queriesPerKvGroup,
                                         static_cast<int32_t>(kvLayout)));
}

// onHost/nn/softmax.hpp:26-40
template <typename T_Type>
void softmax(auto& queue, auto /*exec*/, auto const& input, auto& output, uint32_t axis) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto i = d::to_ann(input), o = d::to_ann(output);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_softmax_f32(d::stream_of(queue), &i, &o, axis));
    else
        d::check(ann_softmax_f64(d::stream_of(queue), &i, &o, axis));
}

// onHost/nn/softmax.hpp:59-80
template <typename T_Type>
void causalSoftmax(auto& queue, auto /*exec*/, auto const& input, auto& output, uint32_t axis, uint32_t queryAxis,
                   uint32_t keyAxis) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto i = d::to_ann(input), o = d::to_ann(output);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_causal_softmax_f32(d::stream_of(queue), &i, &o, axis, queryAxis, keyAxis));
    else
        d::check(ann_causal_softmax_f64(d::stream_of(queue), &i, &o, axis, queryAxis, keyAxis));
}

// onHost/nn/softmax.hpp:42-57
template <typename T_Type>
void maskedSoftmax(auto& queue, auto /*exec*/, auto const& input, auto const& mask, auto& output, uint32_t axis) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto i = d::to_ann(input), m = d::to_ann(mask), o = d::to_ann(output);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_masked_softmax_f32(d::stream_of(queue), &i, &m, &o, axis));
    else
        d::check(ann_masked_softmax_f64(d::stream_of(queue), &i, &m, &o, axis));
}

// ---- MLP layers: onHost/nn/mlp.hpp --------------------------------------------
// :33-37
template <typename T_Type>
void linear(auto& queue, auto const& input, auto const& weight, auto& output) {
    alpaka::nn::onHost::gemm<T_Type>(queue, input, weight, output);
}

// :52-58
enum class Activation { none = ANN_ACT_NONE, relu = ANN_ACT_RELU, silu = ANN_ACT_SILU, gelu = ANN_ACT_GELU };

// :60-76
template <typename T_View>
struct WeightView {
    T_View view;
};
template <typename T_View>
struct BiasView {
    T_View view;
};

// :42-47, the bias add and an optional activation in one pass after the GEMM
template <typename T_Type>
void linearBias(auto& queue, auto /*exec*/, auto const& input, auto const& weight, auto const& bias, auto& output,
                Activation activation = Activation::none) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto i = d::to_ann(input), w = d::to_ann(weight), b = d::to_ann(bias), o = d::to_ann(output);
    int32_t const act = static_cast<int32_t>(activation);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_linear_bias_f32(d::stream_of(queue), &i, &w, &b, act, &o));
    else
        d::check(ann_linear_bias_f64(d::stream_of(queue), &i, &w, &b, act, &o));
}

// :150-218 (hidden / last activation), scratch from a stream-ordered allocation
template <typename T_Type, typename T_WeightView, typename T_BiasView>
void mlpForward(auto& queue, auto /*exec*/, auto const& input, std::span<WeightView<T_WeightView> const> weights,
                std::span<BiasView<T_BiasView> const> biases, Activation hiddenActivation, Activation lastActivation,
                auto& output) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    if (weights.empty()) throw std::invalid_argument{"mlpForward: at least one layer is required."};
    if (weights.size() != biases.size())
        throw std::invalid_argument{"mlpForward: weights and biases must have the same length."};
    std::vector<ann_view> w, b;
    for (auto const& x : weights) w.push_back(d::to_ann(x.view));
    for (auto const& x : biases) b.push_back(d::to_ann(x.view));
    auto i = d::to_ann(input), o = d::to_ann(output);
    int32_t const n = static_cast<int32_t>(w.size());
    int32_t const ha = static_cast<int32_t>(hiddenActivation), la = static_cast<int32_t>(lastActivation);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_mlp_forward_f32(d::stream_of(queue), &i, n, w.data(), b.data(), ha, la, &o, nullptr, 0));
    else
        d::check(ann_mlp_forward_f64(d::stream_of(queue), &i, n, w.data(), b.data(), ha, la, &o, nullptr, 0));
}
// :141-148 (one activation for every layer)
template <typename T_Type, typename T_WeightView, typename T_BiasView>
void mlpForward(auto& queue, auto exec, auto const& input, std::span<WeightView<T_WeightView> const> weights,
                std::span<BiasView<T_BiasView> const> biases, Activation activation, auto& output) {
    mlpForward<T_Type>(queue, exec, input, weights, biases, activation, activation, output);
}
// :248-275 (compile-time depth)
template <typename T_Type, typename T_WeightView, typename T_BiasView, std::size_t T_Depth>
void mlpForward(auto& queue, auto exec, auto const& input, std::array<WeightView<T_WeightView>, T_Depth> const& weights,
                std::array<BiasView<T_BiasView>, T_Depth> const& biases, Activation hiddenActivation,
                Activation lastActivation, auto& output) {
    mlpForward<T_Type>(queue, exec, input, std::span<WeightView<T_WeightView> const>{weights},
                       std::span<BiasView<T_BiasView> const>{biases}, hiddenActivation, lastActivation, output);
}
template <typename T_Type, typename T_WeightView, typename T_BiasView, std::size_t T_Depth>
void mlpForward(auto& queue, auto exec, auto const& input, std::array<WeightView<T_WeightView>, T_Depth> const& weights,
                std::array<BiasView<T_BiasView>, T_Depth> const& biases, Activation activation, auto& output) {
    mlpForward<T_Type>(queue, exec, input, weights, biases, activation, activation, output);
}

// :277-282
template <typename T_Type>
void decodeLatent(auto& queue, auto /*exec*/, auto const& latent, auto const& weight, auto& output) {
    alpaka::nn::onHost::gemm<T_Type>(queue, latent, weight, output);
}

// :307-337, the gated MLP; scratch from a stream-ordered allocation
template <typename T_Type>
void mlp(auto& queue, auto /*exec*/, auto const& input, auto const& Wgate, auto const& Wup, auto const& Wdown,
         auto& output) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto i = d::to_ann(input), g = d::to_ann(Wgate), u = d::to_ann(Wup), w = d::to_ann(Wdown), o = d::to_ann(output);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_mlp_f32(d::stream_of(queue), &i, &g, &u, &w, &o, nullptr, 0));
    else
        d::check(ann_mlp_f64(d::stream_of(queue), &i, &g, &u, &w, &o, nullptr, 0));
}

// onHost/nn/rope.hpp:49-62
template <typename T_Type>
void rope(auto& queue, auto /*exec*/, auto const& in, auto const& cosTable, auto const& sinTable, auto& out,
          alpaka::nn::RopeLayout layout = alpaka::nn::RopeLayout::BTHD, uint32_t positionOffset = 0u) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto i = d::to_ann(in), c = d::to_ann(cosTable), s = d::to_ann(sinTable), o = d::to_ann(out);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_rope_f32(d::stream_of(queue), &i, &c, &s, &o, static_cast<int32_t>(layout), positionOffset));
    else
        d::check(ann_rope_f64(d::stream_of(queue), &i, &c, &s, &o, static_cast<int32_t>(layout), positionOffset));
}

// onHost/nn/rope.hpp:64-86 (query/key overload)
template <typename T_Type>
void rope(auto& queue, auto exec, auto const& q, auto const& k, auto const& cosTable, auto const& sinTable, auto& outQ,
          auto& outK, alpaka::nn::RopeLayout layout = alpaka::nn::RopeLayout::BTHD, uint32_t positionOffset = 0u) {
    rope<T_Type>(queue, exec, q, cosTable, sinTable, outQ, layout, positionOffset);
    rope<T_Type>(queue, exec, k, cosTable, sinTable, outK, layout, positionOffset);
}

// onHost/nn/rope.hpp:96-113 -- truly in place, no temporary
template <typename T_Type>
void ropeInPlace(auto& queue, auto /*exec*/, auto& tensor, auto const& cosTable, auto const& sinTable,
                 alpaka::nn::RopeLayout layout = alpaka::nn::RopeLayout::BTHD, uint32_t positionOffset = 0u) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto t = d::to_ann(tensor), c = d::to_ann(cosTable), s = d::to_ann(sinTable);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_rope_inplace_f32(d::stream_of(queue), &t, nullptr, &c, &s, static_cast<int32_t>(layout),
                                      positionOffset));
    else
        d::check(ann_rope_inplace_f64(d::stream_of(queue), &t, nullptr, &c, &s, static_cast<int32_t>(layout),
                                      positionOffset));
}

// onHost/nn/rope.hpp:122-135 -- q and k rotated in one launch
template <typename T_Type>
void ropeInPlace(auto& queue, auto /*exec*/, auto& q, auto& k, auto const& cosTable, auto const& sinTable,
                 alpaka::nn::RopeLayout layout = alpaka::nn::RopeLayout::BTHD, uint32_t positionOffset = 0u) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto qa = d::to_ann(q), ka = d::to_ann(k), c = d::to_ann(cosTable), s = d::to_ann(sinTable);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_rope_inplace_f32(d::stream_of(queue), &qa, &ka, &c, &s, static_cast<int32_t>(layout),
                                      positionOffset));
    else
        d::check(ann_rope_inplace_f64(d::stream_of(queue), &qa, &ka, &c, &s, static_cast<int32_t>(layout),
                                      positionOffset));
}

// Fused decode: attentionScores -> ops::scale -> softmax -> attentionApply in one kernel.
template <typename T_Type>
void attentionDecode(auto& queue, auto /*exec*/, auto const& Q, auto const& K, auto const& V, auto& out,
                     T_Type scale, uint32_t queriesPerKvGroup = 1u,
                     alpaka::nn::AttentionKvLayout kvLayout = alpaka::nn::AttentionKvLayout::BHTD) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto q = d::to_ann(Q), k = d::to_ann(K), v = d::to_ann(V), o = d::to_ann(out);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_attention_decode_f32(d::stream_of(queue), &q, &k, &v, &o, scale, queriesPerKvGroup,
                                          static_cast<int32_t>(kvLayout)));
    else
        d::check(ann_attention_decode_f64(d::stream_of(queue), &q, &k, &v, &o, scale, queriesPerKvGroup,
                                          static_cast<int32_t>(kvLayout)));
}

// Fused prefill: attentionScores -> ops::scale -> causalSoftmax / softmax -> attentionApply in one kernel.
template <typename T_Type>
void attentionPrefill(auto& queue, auto /*exec*/, auto const& Q, auto const& K, auto const& V, auto& out,
                      T_Type scale, uint32_t queriesPerKvGroup = 1u,
                      alpaka::nn::AttentionKvLayout kvLayout = alpaka::nn::AttentionKvLayout::BTHD,
                      bool causal = true) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto q = d::to_ann(Q), k = d::to_ann(K), v = d::to_ann(V), o = d::to_ann(out);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_attention_prefill_f32(d::stream_of(queue), &q, &k, &v, &o, scale, queriesPerKvGroup,
                                           static_cast<int32_t>(kvLayout), causal ? 1 : 0));
    else
        d::check(ann_attention_prefill_f64(d::stream_of(queue), &q, &k, &v, &o, scale, queriesPerKvGroup,
                                           static_cast<int32_t>(kvLayout), causal ? 1 : 0));
}

// attentionDecode / attentionPrefill whose result stores go through `outMirror`,
// the NVLink multicast address of out's first element, into every rank's copy
// of the output (include/ann_b200.h, multicast outputs); enqueue
// b200::signalBarrier after them on every rank.
template <typename T_Type>
void attentionDecodeMirror(auto& queue, auto /*exec*/, auto const& Q, auto const& K, auto const& V, auto& out,
                           void* outMirror, T_Type scale, uint32_t queriesPerKvGroup = 1u,
                           alpaka::nn::AttentionKvLayout kvLayout = alpaka::nn::AttentionKvLayout::BHTD) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto q = d::to_ann(Q), k = d::to_ann(K), v = d::to_ann(V), o = d::to_ann(out);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_attention_decode_mirror_f32(d::stream_of(queue), &q, &k, &v, &o, outMirror, scale,
                                                 queriesPerKvGroup, static_cast<int32_t>(kvLayout)));
    else
        d::check(ann_attention_decode_mirror_f64(d::stream_of(queue), &q, &k, &v, &o, outMirror, scale,
                                                 queriesPerKvGroup, static_cast<int32_t>(kvLayout)));
}

template <typename T_Type>
void attentionPrefillMirror(auto& queue, auto /*exec*/, auto const& Q, auto const& K, auto const& V, auto& out,
                            void* outMirror, T_Type scale, uint32_t queriesPerKvGroup = 1u,
                            alpaka::nn::AttentionKvLayout kvLayout = alpaka::nn::AttentionKvLayout::BTHD,
                            bool causal = true) {
    namespace d = alpaka::nn::b200::detail;
    d::require_float<T_Type>();
    auto q = d::to_ann(Q), k = d::to_ann(K), v = d::to_ann(V), o = d::to_ann(out);
    if constexpr (d::is_f32<T_Type>)
        d::check(ann_attention_prefill_mirror_f32(d::stream_of(queue), &q, &k, &v, &o, outMirror, scale,
                                                  queriesPerKvGroup, static_cast<int32_t>(kvLayout), causal ? 1 : 0));
    else
        d::check(ann_attention_prefill_mirror_f64(d::stream_of(queue), &q, &k, &v, &o, outMirror, scale,
                                                  queriesPerKvGroup, static_cast<int32_t>(kvLayout), causal ? 1 : 0));
}

}  // namespace alpaka::nn::onHost::nn

namespace alpaka::nn::b200 {

// Cross-rank barrier over peer-addressable signal words (ann_signal_barrier):
// epochs 1, 2, 3, ... in the same order on every rank; a wait that runs out
// sets ANN_DEVERR_WAIT_TIMEOUT (ann_take_device_error).
template <typename Q>
void signalBarrier(Q& queue, uint32_t* signals, uint32_t* const* peerSignals, int nranks, int rank, uint32_t epoch,
                   uint64_t timeoutNs = 5000000000ull) {
    detail::check(ann_signal_barrier(detail::stream_of(queue), signals, peerSignals, nranks, rank, epoch, timeoutNs));
}

// The same barrier with its epoch in device memory (ann_signal_barrier_dev):
// `epochWord` (zero before the first call) advances on the device, so the call
// can be captured in a CUDA graph and replayed.
template <typename Q>
void signalBarrierDev(Q& queue, uint32_t* signals, uint32_t* const* peerSignals, int nranks, int rank,
                      uint32_t* epochWord, uint64_t timeoutNs = 5000000000ull) {
    detail::check(
        ann_signal_barrier_dev(detail::stream_of(queue), signals, peerSignals, nranks, rank, epochWord, timeoutNs));
}

// One rank of the node's NCCL communicator (ann_comm_*), on the current CUDA
// device. Rank 0 creates the rendezvous id with uniqueId() and hands its bytes
// to the other ranks out of band; a rank whose peers do not all join within
// timeoutSeconds gets std::runtime_error (ANN_ENCCL) instead of waiting for good.
class Comm {
public:
    using Id = std::array<unsigned char, ANN_COMM_ID_BYTES>;

    static Id uniqueId() {
        Id id{};
        detail::check(ann_comm_unique_id(id.data()));
        return id;
    }
    Comm(int nranks, int rank, Id const& id, double timeoutSeconds = 60.0) {
        detail::check(ann_comm_init(&comm_, nranks, rank, id.data(), timeoutSeconds));
        nranks_ = nranks;
        rank_ = rank;
    }
    Comm(Comm const&) = delete;
    Comm& operator=(Comm const&) = delete;
    ~Comm() {
        if (comm_) ann_comm_destroy(comm_);
    }
    int size() const { return nranks_; }
    int rank() const { return rank_; }

    // recv = the bytesPerRank of every rank's send, rank-major, enqueued on queue.
    template <typename Q>
    void allGather(Q& queue, void const* send, void* recv, std::size_t bytesPerRank) {
        detail::check(ann_comm_allgather(comm_, detail::stream_of(queue), send, recv, bytesPerRank));
    }
    // Tear down at once (a peer died); the destructor then does nothing.
    void abort() {
        if (comm_) ann_comm_abort(comm_);
        comm_ = nullptr;
    }

private:
    ann_comm comm_ = nullptr;
    int nranks_ = 0, rank_ = 0;
};

// One decode step of the head-sharded path on this rank of comm: RoPE on q and
// the new K row, fused decode over this rank's cache slice into outLocal
// [B,1,H/G,D], all-gather into gathered [G,B,1,H/G,D] (rank-major), re-assembly
// into out [B,1,H,D] (BTHD). All views dense; caches BHTD [B,H_kv/G,Tk,D].
template <typename T_Type>
void headShardedDecode(auto& queue, Comm& comm, View<T_Type, 4>& q, View<T_Type, 4>& knew,
                       auto const& cosTable, auto const& sinTable, uint32_t position,
                       View<T_Type, 4> const& kCache, View<T_Type, 4> const& vCache, View<T_Type, 4>& outLocal,
                       View<T_Type, 5>& gathered, View<T_Type, 4>& out, T_Type scale, uint32_t queriesPerKvGroup = 1u) {
    onHost::nn::ropeInPlace<T_Type>(queue, 0, q, knew, cosTable, sinTable, RopeLayout::BTHD, position);
    onHost::nn::attentionDecode<T_Type>(queue, 0, q, kCache, vCache, outLocal, scale, queriesPerKvGroup,
                                        AttentionKvLayout::BHTD);
    auto const& le = outLocal.extents;
    std::size_t const bytes = static_cast<std::size_t>(le[0] * le[1] * le[2] * le[3]) * sizeof(T_Type);
    comm.allGather(queue, outLocal.data(), gathered.data(), bytes);
    // gathered[r, b, t, h, d] -> out[b, t, r * H/G + h, d]: two strided 5-D views of the same order
    View<T_Type, 5> src;
    src.ptr = gathered.ptr;
    src.extents = {gathered.extents[1], gathered.extents[2], gathered.extents[0], gathered.extents[3],
                   gathered.extents[4]};
    src.pitches = {gathered.pitches[1], gathered.pitches[2], gathered.pitches[0], gathered.pitches[3],
                   gathered.pitches[4]};
    View<T_Type, 5> dst;
    dst.ptr = out.ptr;
    dst.extents = src.extents;
    dst.pitches = {out.pitches[0], out.pitches[1], out.pitches[2] * gathered.extents[3], out.pitches[2],
                   out.pitches[3]};
    onHost::ops::scale<T_Type>(queue, 0, src, T_Type(1), dst);
}

}  // namespace alpaka::nn::b200
