// ops.cu -- elementwise ops, activations, bias add, cast / fill and axis
// reductions (reference: onHost/ops/elementwise.hpp, onHost/ops/reduction.hpp).
//
// All of these are HBM-bound: one read of each operand, one write.
//  - Elementwise: when every operand is a dense row-major tensor of the same
//    extents the grid walks a flat index, with 16-byte vector loads/stores
//    when every pointer is 16-byte aligned (a scalar loop takes the tail);
//    otherwise a strided walk over up to 8 axes with byte pitches, the
//    reference's arbitrary views.
//  - Arithmetic keeps the reference's expression order with uncontracted
//    multiplies and adds (no FMA), so copy/scale/add/sub/mul/div/axpy/relu/
//    sqrt/biasAdd/cast are bit-identical to a host loop; exp/erf-based ones
//    (exp, sigmoid, silu, gelu, swiglu) and rsqrt differ only by the device
//    math functions' last-place error.
//  - biasAdd + activation fuse into one pass (the reference's mlpForward runs
//    biasAdd, then the activation in place: two passes with the same two
//    roundings).
//  - Reductions: a row along a unit-stride axis is reduced by a warp with
//    16-byte loads, four in flight per lane, when the rows are 16-byte
//    aligned (else a warp or a 256-thread CTA with element loads); any other
//    axis by 32 adjacent outputs per CTA, eight warps splitting the axis, so
//    the loads of a warp are adjacent in memory whenever the output's last
//    axis is -- and when those tiles are too few to fill the GPU, by a
//    cluster of eight CTAs per tile that split the axis and combine through
//    distributed shared memory.
#include <cooperative_groups.h>

#include <cstring>

#include "common.cuh"
#include "reduce.cuh"

namespace cg = cooperative_groups;

namespace ann {
namespace {

// ---------------------------------------------------------------------------
// Operators (elementwise.hpp:15-178)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float erf_t(float x) { return erff(x); }
__device__ __forceinline__ double erf_t(double x) { return erf(x); }
__device__ __forceinline__ float sqrt_t(float x) { return sqrtf(x); }
__device__ __forceinline__ double sqrt_t(double x) { return sqrt(x); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ double div_rn(double a, double b) { return __ddiv_rn(a, b); }

template <typename T>
__device__ __forceinline__ T sigmoid_of(T x) {  // 1 / (1 + exp(-x))
    return div_rn(T(1), add_rn(T(1), exp_t(-x)));
}

template <int OP, typename T>
__device__ __forceinline__ T unary(T x, T s) {
    if constexpr (OP == ANN_UNARY_COPY) return x;
    else if constexpr (OP == ANN_UNARY_SCALE) return mul_rn(x, s);
    else if constexpr (OP == ANN_UNARY_EXP) return exp_t(x);
    else if constexpr (OP == ANN_UNARY_SQRT) return sqrt_t(x);
    else if constexpr (OP == ANN_UNARY_RSQRT) return rsqrt_t(x);
    else if constexpr (OP == ANN_UNARY_RELU) return x > T(0) ? x : T(0);
    else if constexpr (OP == ANN_UNARY_SIGMOID) return sigmoid_of(x);
    else if constexpr (OP == ANN_UNARY_SILU) return mul_rn(x, sigmoid_of(x));
    else {  // GELU: 0.5 * x * (1 + erf(x * 1/sqrt(2)))
        T const inv_sqrt2 = static_cast<T>(0.70710678118654752440);
        return mul_rn(mul_rn(T(0.5), x), add_rn(T(1), erf_t(mul_rn(x, inv_sqrt2))));
    }
}

template <int OP, typename T>
__device__ __forceinline__ T binary(T l, T r, T alpha) {
    if constexpr (OP == ANN_BINARY_ADD) return add_rn(l, r);
    else if constexpr (OP == ANN_BINARY_SUB) return sub_rn(l, r);
    else if constexpr (OP == ANN_BINARY_MUL) return mul_rn(l, r);
    else if constexpr (OP == ANN_BINARY_DIV) return div_rn(l, r);
    else if constexpr (OP == ANN_BINARY_AXPY) return add_rn(mul_rn(alpha, l), r);
    else return mul_rn(mul_rn(l, sigmoid_of(l)), r);  // SWIGLU: lhs * sigmoid(lhs) * rhs
}

// Activation after a bias add (mlp.hpp:52-58, 82-103); NONE is plain biasAdd.
template <int ACT, typename T>
__device__ __forceinline__ T activate(T v) {
    if constexpr (ACT == ANN_ACT_NONE) return v;
    else if constexpr (ACT == ANN_ACT_RELU) return unary<ANN_UNARY_RELU>(v, T(0));
    else if constexpr (ACT == ANN_ACT_SILU) return unary<ANN_UNARY_SILU>(v, T(0));
    else return unary<ANN_UNARY_GELU>(v, T(0));
}

// ---------------------------------------------------------------------------
// Index walks
// ---------------------------------------------------------------------------
// Element offsets of up to three tensors that share extents.
struct Walk3 {
    int n = 0;
    int64_t ext[ANN_MAX_RANK] = {};
    int64_t s[3][ANN_MAX_RANK] = {};
    __device__ __forceinline__ void offsets(int64_t flat, int64_t& o0, int64_t& o1, int64_t& o2) const {
        o0 = o1 = o2 = 0;
        for (int a = n - 1; a >= 0; --a) {
            int64_t const i = flat % ext[a];
            flat /= ext[a];
            o0 += i * s[0][a];
            o1 += i * s[1][a];
            o2 += i * s[2][a];
        }
    }
};

Walk3 walk_of(const Dims& shape, const Dims* t0, const Dims* t1, const Dims* t2) {
    Walk3 w;
    w.n = shape.rank;
    for (int a = 0; a < shape.rank; ++a) {
        w.ext[a] = shape.ext[a];
        w.s[0][a] = t0 ? t0->str[a] : 0;
        w.s[1][a] = t1 ? t1->str[a] : 0;
        w.s[2][a] = t2 ? t2->str[a] : 0;
    }
    return w;
}

constexpr int kThreads = 256;

inline int blocks_for(int64_t n, int per_thread) {
    return grid_for(ceil_div(n, per_thread), kThreads, 8);
}

// ---- unary / binary / bias: dense and strided kernels ----------------------
// Dense: elements [0, n) of flat arrays; 16-byte vectors when vec_ok (every
// pointer 16-byte aligned), the remainder element by element.
template <int OP, typename T>
__global__ void __launch_bounds__(kThreads) unary_dense(T const* in, T* out, int64_t n,
                                                        T s, int vec_ok) {
    using V = typename Vec16<T>::type;
    constexpr int NV = Vec16<T>::n;
    int64_t const tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    int64_t const stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    int64_t done = 0;
    if (vec_ok) {
        int64_t const nv = n / NV;
        V const* vi = reinterpret_cast<V const*>(in);
        V* vo = reinterpret_cast<V*>(out);
        for (int64_t i = tid; i < nv; i += stride) {
            V x = vi[i];
            T* e = reinterpret_cast<T*>(&x);
#pragma unroll
            for (int k = 0; k < NV; ++k) e[k] = unary<OP>(e[k], s);
            vo[i] = x;
        }
        done = nv * NV;
    }
    for (int64_t i = done + tid; i < n; i += stride) out[i] = unary<OP>(in[i], s);
}

template <int OP, typename T>
__global__ void __launch_bounds__(kThreads) unary_strided(T const* in, T* out, int64_t n, Walk3 w, T s) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t oo, oi, unused;
        w.offsets(i, oo, oi, unused);
        out[oo] = unary<OP>(in[oi], s);
    }
}

template <int OP, typename T>
__global__ void __launch_bounds__(kThreads) binary_dense(T const* l, T const* r,
                                                         T* out, int64_t n, T alpha, int vec_ok) {
    using V = typename Vec16<T>::type;
    constexpr int NV = Vec16<T>::n;
    int64_t const tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    int64_t const stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    int64_t done = 0;
    if (vec_ok) {
        int64_t const nv = n / NV;
        V const* vl = reinterpret_cast<V const*>(l);
        V const* vr = reinterpret_cast<V const*>(r);
        V* vo = reinterpret_cast<V*>(out);
        auto apply = [&](V a, V const& b) {
            T* ea = reinterpret_cast<T*>(&a);
            T const* eb = reinterpret_cast<T const*>(&b);
#pragma unroll
            for (int k = 0; k < NV; ++k) ea[k] = binary<OP>(ea[k], eb[k], alpha);
            return a;
        };
        int64_t i = tid;
        for (; i + stride < nv; i += 2 * stride) {  // four loads in flight
            V const a0 = vl[i], b0 = vr[i], a1 = vl[i + stride], b1 = vr[i + stride];
            vo[i] = apply(a0, b0);
            vo[i + stride] = apply(a1, b1);
        }
        if (i < nv) vo[i] = apply(vl[i], vr[i]);
        done = nv * NV;
    }
    for (int64_t i = done + tid; i < n; i += stride) out[i] = binary<OP>(l[i], r[i], alpha);
}

template <int OP, typename T>
__global__ void __launch_bounds__(kThreads) binary_strided(T const* l, T const* r, T* out, int64_t n, Walk3 w,
                                                           T alpha) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t oo, ol, orr;
        w.offsets(i, oo, ol, orr);
        out[oo] = binary<OP>(l[ol], r[orr], alpha);
    }
}

// out[..., h] = act(in[..., h] + bias[h]); dense rows of length H.
// FIXED_COL: the grid stride is a whole number of rows, so every vector a
// thread touches has the same column: its bias vector is loaded once. Four
// vectors per thread per iteration keep four loads in flight.
template <int ACT, typename T, bool FIXED_COL>
__global__ void __launch_bounds__(kThreads) bias_dense(T const* in, T const* bias, T* out, int64_t n, int64_t H,
                                                       int vec_ok) {
    using V = typename Vec16<T>::type;
    constexpr int NV = Vec16<T>::n;
    int64_t const tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    int64_t const stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    if (vec_ok) {  // H % NV == 0: a vector never straddles two rows
        int64_t const nv = n / NV, hv = H / NV;
        V const* vi = reinterpret_cast<V const*>(in);
        V const* vb = reinterpret_cast<V const*>(bias);
        V* vo = reinterpret_cast<V*>(out);
        auto apply = [](V x, V const& b) {
            T* e = reinterpret_cast<T*>(&x);
            T const* eb = reinterpret_cast<T const*>(&b);
#pragma unroll
            for (int k = 0; k < NV; ++k) e[k] = activate<ACT>(add_rn(e[k], eb[k]));
            return x;
        };
        if constexpr (FIXED_COL) {
            V const b = vb[tid % hv];
            int64_t i = tid;
            for (; i + 3 * stride < nv; i += 4 * stride) {
                V const x0 = vi[i], x1 = vi[i + stride], x2 = vi[i + 2 * stride], x3 = vi[i + 3 * stride];
                vo[i] = apply(x0, b);
                vo[i + stride] = apply(x1, b);
                vo[i + 2 * stride] = apply(x2, b);
                vo[i + 3 * stride] = apply(x3, b);
            }
            for (; i < nv; i += stride) vo[i] = apply(vi[i], b);
        } else {
            // column of vector i, advanced by the stride's remainder each
            // iteration instead of a 64-bit modulo per vector
            int64_t col = tid % hv;
            int64_t const step = stride % hv;
            for (int64_t i = tid; i < nv; i += stride) {
                vo[i] = apply(vi[i], vb[col]);
                col += step;
                if (col >= hv) col -= hv;
            }
        }
        return;
    }
    for (int64_t i = tid; i < n; i += stride) out[i] = activate<ACT>(add_rn(in[i], bias[i % H]));
}

template <int ACT, typename T>
__global__ void __launch_bounds__(kThreads) bias_strided(T const* in, T const* bias, int64_t bias_stride, T* out,
                                                         int64_t n, Walk3 w) {
    int const last = w.n - 1;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t oo, oi, unused;
        w.offsets(i, oo, oi, unused);
        out[oo] = activate<ACT>(add_rn(in[oi], bias[(i % w.ext[last]) * bias_stride]));
    }
}

// ---------------------------------------------------------------------------
// Host dispatch
// ---------------------------------------------------------------------------
bool dense_alike(const Dims& a, const Dims& b) {
    if (!same_extents(a, b) || !a.dense() || !b.dense()) return false;
    return true;
}

inline bool vec_aligned(const void* p) { return aligned(p, 16); }

template <typename T, int OP>
void launch_unary(cudaStream_t s, const Dims& in, const Dims& out, T scalar) {
    int64_t const n = out.numel();
    if (dense_alike(in, out)) {
        int const vec = vec_aligned(in.data) && vec_aligned(out.data);
        unary_dense<OP, T><<<blocks_for(n, vec ? Vec16<T>::n : 1), kThreads, 0, s>>>(
            static_cast<T const*>(in.data), static_cast<T*>(out.data), n, scalar, vec);
    } else {
        unary_strided<OP, T><<<blocks_for(n, 1), kThreads, 0, s>>>(
            static_cast<T const*>(in.data), static_cast<T*>(out.data), n, walk_of(out, &out, &in, nullptr), scalar);
    }
}

template <typename T>
int unary_op(ann_stream stream, int op, const ann_view* in_v, const ann_view* out_v, T scalar) {
    Dims in, out;
    ANN_TRY(to_dims(in_v, sizeof(T), "unaryOp input", in));
    ANN_TRY(to_dims(out_v, sizeof(T), "unaryOp output", out));
    char const* name = op == ANN_UNARY_COPY ? "copy" : "unaryOp";  // elementwise.hpp:260, 279
    if (!same_extents(in, out)) return fail(ANN_EINVAL, "%s shape mismatch.", name);
    if (op < ANN_UNARY_COPY || op > ANN_UNARY_GELU) return fail(ANN_EINVAL, "unaryOp: unknown operator %d.", op);
    if (out.numel() == 0) return ANN_OK;
    cudaStream_t s = as_stream(stream);
    switch (op) {
        case ANN_UNARY_COPY: launch_unary<T, ANN_UNARY_COPY>(s, in, out, scalar); break;
        case ANN_UNARY_SCALE: launch_unary<T, ANN_UNARY_SCALE>(s, in, out, scalar); break;
        case ANN_UNARY_EXP: launch_unary<T, ANN_UNARY_EXP>(s, in, out, scalar); break;
        case ANN_UNARY_SQRT: launch_unary<T, ANN_UNARY_SQRT>(s, in, out, scalar); break;
        case ANN_UNARY_RSQRT: launch_unary<T, ANN_UNARY_RSQRT>(s, in, out, scalar); break;
        case ANN_UNARY_RELU: launch_unary<T, ANN_UNARY_RELU>(s, in, out, scalar); break;
        case ANN_UNARY_SIGMOID: launch_unary<T, ANN_UNARY_SIGMOID>(s, in, out, scalar); break;
        case ANN_UNARY_SILU: launch_unary<T, ANN_UNARY_SILU>(s, in, out, scalar); break;
        default: launch_unary<T, ANN_UNARY_GELU>(s, in, out, scalar); break;
    }
    return check_launch("unaryOp");
}

template <typename T, int OP>
void launch_binary(cudaStream_t s, const Dims& l, const Dims& r, const Dims& out, T alpha) {
    int64_t const n = out.numel();
    if (dense_alike(l, out) && dense_alike(r, out)) {
        int const vec = vec_aligned(l.data) && vec_aligned(r.data) && vec_aligned(out.data);
        binary_dense<OP, T><<<blocks_for(n, vec ? Vec16<T>::n : 1), kThreads, 0, s>>>(
            static_cast<T const*>(l.data), static_cast<T const*>(r.data), static_cast<T*>(out.data), n, alpha, vec);
    } else {
        binary_strided<OP, T><<<blocks_for(n, 1), kThreads, 0, s>>>(
            static_cast<T const*>(l.data), static_cast<T const*>(r.data), static_cast<T*>(out.data), n,
            walk_of(out, &out, &l, &r), alpha);
    }
}

template <typename T>
int binary_op(ann_stream stream, int op, const ann_view* l_v, const ann_view* r_v, const ann_view* out_v, T alpha) {
    Dims l, r, out;
    ANN_TRY(to_dims(l_v, sizeof(T), "binaryOp lhs", l));
    ANN_TRY(to_dims(r_v, sizeof(T), "binaryOp rhs", r));
    ANN_TRY(to_dims(out_v, sizeof(T), "binaryOp output", out));
    if (!same_extents(l, r) || !same_extents(l, out)) return fail(ANN_EINVAL, "binaryOp shape mismatch.");
    if (op < ANN_BINARY_ADD || op > ANN_BINARY_SWIGLU) return fail(ANN_EINVAL, "binaryOp: unknown operator %d.", op);
    if (out.numel() == 0) return ANN_OK;
    cudaStream_t s = as_stream(stream);
    switch (op) {
        case ANN_BINARY_ADD: launch_binary<T, ANN_BINARY_ADD>(s, l, r, out, alpha); break;
        case ANN_BINARY_SUB: launch_binary<T, ANN_BINARY_SUB>(s, l, r, out, alpha); break;
        case ANN_BINARY_MUL: launch_binary<T, ANN_BINARY_MUL>(s, l, r, out, alpha); break;
        case ANN_BINARY_DIV: launch_binary<T, ANN_BINARY_DIV>(s, l, r, out, alpha); break;
        case ANN_BINARY_AXPY: launch_binary<T, ANN_BINARY_AXPY>(s, l, r, out, alpha); break;
        default: launch_binary<T, ANN_BINARY_SWIGLU>(s, l, r, out, alpha); break;
    }
    return check_launch("binaryOp");
}

template <typename T, int ACT>
void launch_bias(cudaStream_t s, const Dims& in, const Dims& bias, const Dims& out) {
    int64_t const n = out.numel();
    int64_t const H = out.ext[out.rank - 1];
    if (dense_alike(in, out) && bias.str[0] == 1) {
        int const vec = vec_aligned(in.data) && vec_aligned(out.data) && vec_aligned(bias.data) &&
                        H % Vec16<T>::n == 0;
        int grid = blocks_for(n, vec ? Vec16<T>::n : 1);
        T const* pi = static_cast<T const*>(in.data);
        T const* pb = static_cast<T const*>(bias.data);
        T* po = static_cast<T*>(out.data);
        if (vec) {
            // A grid whose stride (grid * kThreads vectors) is a multiple of
            // the row's hv vectors keeps each thread on one column.
            int64_t const hv = H / Vec16<T>::n;
            int64_t g = hv, t = kThreads;  // g = hv / gcd(hv, kThreads)
            while (t != 0) {
                int64_t const r = g % t;
                g = t;
                t = r;
            }
            int64_t const period = hv / g;
            if (period <= grid) {
                grid = static_cast<int>(grid / period * period);
                bias_dense<ACT, T, true><<<grid, kThreads, 0, s>>>(pi, pb, po, n, H, 1);
                return;
            }
        }
        bias_dense<ACT, T, false><<<grid, kThreads, 0, s>>>(pi, pb, po, n, H, vec);
    } else {
        bias_strided<ACT, T><<<blocks_for(n, 1), kThreads, 0, s>>>(
            static_cast<T const*>(in.data), static_cast<T const*>(bias.data), bias.str[0], static_cast<T*>(out.data),
            n, walk_of(out, &out, &in, nullptr));
    }
}

// biasAdd (elementwise.hpp:348-366) with an optional fused activation.
template <typename T>
int bias_act(ann_stream stream, const ann_view* in_v, const ann_view* bias_v, int act, const ann_view* out_v) {
    Dims in, bias, out;
    ANN_TRY(to_dims(in_v, sizeof(T), "biasAdd input", in));
    ANN_TRY(to_dims(bias_v, sizeof(T), "biasAdd bias", bias));
    ANN_TRY(to_dims(out_v, sizeof(T), "biasAdd output", out));
    if (!same_extents(in, out)) return fail(ANN_EINVAL, "biasAdd shape mismatch.");
    if (bias.rank != 1) return fail(ANN_EINVAL, "biasAdd expects a 1D bias view.");
    if (bias.ext[0] != in.ext[in.rank - 1]) return fail(ANN_EINVAL, "biasAdd expects bias extent to match the last axis.");
    if (act < ANN_ACT_NONE || act > ANN_ACT_GELU) return fail(ANN_EINVAL, "mlpForward: unsupported activation.");
    if (out.numel() == 0) return ANN_OK;
    cudaStream_t s = as_stream(stream);
    switch (act) {
        case ANN_ACT_NONE: launch_bias<T, ANN_ACT_NONE>(s, in, bias, out); break;
        case ANN_ACT_RELU: launch_bias<T, ANN_ACT_RELU>(s, in, bias, out); break;
        case ANN_ACT_SILU: launch_bias<T, ANN_ACT_SILU>(s, in, bias, out); break;
        default: launch_bias<T, ANN_ACT_GELU>(s, in, bias, out); break;
    }
    return check_launch("biasAdd");
}

// ---- cast / fill -------------------------------------------------------------
size_t dtype_size(int dt) {
    switch (dt) {
        case ANN_DTYPE_F32: case ANN_DTYPE_I32: case ANN_DTYPE_U32: return 4;
        case ANN_DTYPE_F64: case ANN_DTYPE_I64: return 8;
        default: return 0;
    }
}

template <typename O, typename I>
__global__ void __launch_bounds__(kThreads) cast_kernel(I const* in, O* out, int64_t n, Walk3 w, int dense) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t oo = i, oi = i, unused;
        if (!dense) w.offsets(i, oo, oi, unused);
        out[oo] = static_cast<O>(in[oi]);
    }
}

template <typename O>
void cast_from(cudaStream_t s, int in_dt, const Dims& in, const Dims& out, int dense) {
    int64_t const n = out.numel();
    Walk3 const w = walk_of(out, &out, &in, nullptr);
    O* o = static_cast<O*>(out.data);
    int const g = blocks_for(n, 1);
    switch (in_dt) {
        case ANN_DTYPE_F32: cast_kernel<O, float><<<g, kThreads, 0, s>>>(static_cast<float const*>(in.data), o, n, w, dense); break;
        case ANN_DTYPE_F64: cast_kernel<O, double><<<g, kThreads, 0, s>>>(static_cast<double const*>(in.data), o, n, w, dense); break;
        case ANN_DTYPE_I32: cast_kernel<O, int32_t><<<g, kThreads, 0, s>>>(static_cast<int32_t const*>(in.data), o, n, w, dense); break;
        case ANN_DTYPE_U32: cast_kernel<O, uint32_t><<<g, kThreads, 0, s>>>(static_cast<uint32_t const*>(in.data), o, n, w, dense); break;
        default: cast_kernel<O, int64_t><<<g, kThreads, 0, s>>>(static_cast<int64_t const*>(in.data), o, n, w, dense); break;
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) fill_kernel(T* out, int64_t n, Walk3 w, T value, int dense) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t oo = i, u1, u2;
        if (!dense) w.offsets(i, oo, u1, u2);
        out[oo] = value;
    }
}

template <typename T>
void fill_as(cudaStream_t s, const Dims& out, const void* value) {
    T v;
    std::memcpy(&v, value, sizeof(T));
    int64_t const n = out.numel();
    fill_kernel<T><<<blocks_for(n, 1), kThreads, 0, s>>>(static_cast<T*>(out.data), n,
                                                         walk_of(out, &out, nullptr, nullptr), v, out.dense());
}

// ---- reductions (reduction.hpp:52-289) ----------------------------------------
template <int OP, typename T>
__device__ __forceinline__ T reduce_init() {
    if constexpr (OP == ANN_REDUCE_MAX) return Lowest<T>::value;
    else return T(0);
}
template <int OP, typename T>
__device__ __forceinline__ T transform(T x, T y) {
    if constexpr (OP == ANN_REDUCE_SUM_SQUARES) return mul_rn(x, x);
    else if constexpr (OP == ANN_REDUCE_DOT) return mul_rn(x, y);
    else return x;
}
template <int OP, typename T>
__device__ __forceinline__ T combine(T a, T b) {
    if constexpr (OP == ANN_REDUCE_MAX) return a > b ? a : b;  // MaxReducer
    else return add_rn(a, b);
}
template <int OP, typename T>
__device__ __forceinline__ T finalize(T v, int64_t count) {
    if constexpr (OP == ANN_REDUCE_MEAN) return div_rn(v, static_cast<T>(static_cast<uint32_t>(count)));
    else return v;
}

struct ReduceArgs {
    const void* a;
    const void* b;  // dot's rhs, else unused
    void* out;
    int64_t outputs, len;
    int64_t sa_axis, sb_axis;  // element strides along the reduced axis
    Walk3 w;                   // output extents; strides of out, a, b
};

// One warp per output, the axis unit-stride and every row start 16-byte
// aligned in a (and b): 16-byte loads, four in flight per lane.
template <int OP, typename T>
__global__ void __launch_bounds__(kThreads) reduce_rows_vec(ReduceArgs r) {
    using V = typename Vec16<T>::type;
    constexpr int NV = Vec16<T>::n;
    T const* A = static_cast<T const*>(r.a);
    T const* Bp = static_cast<T const*>(r.b);
    T* out = static_cast<T*>(r.out);
    int const lane = threadIdx.x & 31;
    int64_t const warps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
    int64_t const nv = r.len / NV;
    for (int64_t o = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + threadIdx.x / 32; o < r.outputs;
         o += warps) {
        int64_t oo, oa, ob;
        r.w.offsets(o, oo, oa, ob);
        V const* va = reinterpret_cast<V const*>(A + oa);
        V const* vb = reinterpret_cast<V const*>(Bp + ob);
        T acc = reduce_init<OP, T>();
        int64_t i = lane;
        for (; i + 96 < nv; i += 128) {  // four vectors per lane in flight
            V xa[4], xb[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                xa[u] = va[i + 32 * u];
                if constexpr (OP == ANN_REDUCE_DOT) xb[u] = vb[i + 32 * u];
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                T const* ea = reinterpret_cast<T const*>(&xa[u]);
                T const* eb = reinterpret_cast<T const*>(&xb[u]);
#pragma unroll
                for (int k = 0; k < NV; ++k)
                    acc = combine<OP>(acc, transform<OP>(ea[k], OP == ANN_REDUCE_DOT ? eb[k] : T(0)));
            }
        }
        for (; i < nv; i += 32) {
            V const xa = va[i];
            V xb{};
            if constexpr (OP == ANN_REDUCE_DOT) xb = vb[i];
            T const* ea = reinterpret_cast<T const*>(&xa);
            T const* eb = reinterpret_cast<T const*>(&xb);
#pragma unroll
            for (int k = 0; k < NV; ++k)
                acc = combine<OP>(acc, transform<OP>(ea[k], OP == ANN_REDUCE_DOT ? eb[k] : T(0)));
        }
        for (int64_t e = nv * NV + lane; e < r.len; e += 32)  // tail elements
            acc = combine<OP>(acc, transform<OP>(A[oa + e], OP == ANN_REDUCE_DOT ? Bp[ob + e] : T(0)));
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) acc = combine<OP>(acc, __shfl_xor_sync(0xffffffffu, acc, m));
        if (lane == 0) out[oo] = finalize<OP>(acc, r.len);
    }
}

// One GROUP-thread team per output; the axis has unit stride in a (and b).
template <int OP, typename T, int GROUP>
__global__ void __launch_bounds__(kThreads) reduce_rows(ReduceArgs r) {
    constexpr int TEAMS = kThreads / GROUP;
    __shared__ T scratch[kThreads / 32];
    T const* A = static_cast<T const*>(r.a);
    T const* Bp = static_cast<T const*>(r.b);
    T* out = static_cast<T*>(r.out);
    int const gl = threadIdx.x % GROUP;
    int64_t const iters = ceil_div(r.outputs, static_cast<int64_t>(gridDim.x) * TEAMS);
    for (int64_t it = 0; it < iters; ++it) {
        int64_t const o = (it * gridDim.x + blockIdx.x) * TEAMS + threadIdx.x / GROUP;
        bool const live = o < r.outputs;
        T acc = reduce_init<OP, T>();
        int64_t oo = 0, oa = 0, ob = 0;
        if (live) {
            r.w.offsets(o, oo, oa, ob);
            for (int64_t i = gl; i < r.len; i += GROUP)
                acc = combine<OP>(acc, transform<OP>(A[oa + i], OP == ANN_REDUCE_DOT ? Bp[ob + i] : T(0)));
        }
        if constexpr (GROUP == 32) {
#pragma unroll
            for (int m = 16; m > 0; m >>= 1) acc = combine<OP>(acc, __shfl_xor_sync(0xffffffffu, acc, m));
        } else {
#pragma unroll
            for (int m = 16; m > 0; m >>= 1) acc = combine<OP>(acc, __shfl_xor_sync(0xffffffffu, acc, m));
            if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = acc;
            __syncthreads();
            acc = scratch[0];
            for (int k = 1; k < kThreads / 32; ++k) acc = combine<OP>(acc, scratch[k]);
            __syncthreads();
        }
        if (live && gl == 0) out[oo] = finalize<OP>(acc, r.len);
    }
}

// 32 adjacent outputs per CTA, 8 warps splitting the axis.
template <int OP, typename T>
__global__ void __launch_bounds__(kThreads) reduce_cols(ReduceArgs r) {
    __shared__ T part[8][33];
    T const* A = static_cast<T const*>(r.a);
    T const* Bp = static_cast<T const*>(r.b);
    T* out = static_cast<T*>(r.out);
    int const lane = threadIdx.x & 31, wy = threadIdx.x >> 5;
    int64_t const tiles = ceil_div(r.outputs, 32);
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        int64_t const o = t * 32 + lane;
        T acc = reduce_init<OP, T>();
        int64_t oo = 0, oa = 0, ob = 0;
        if (o < r.outputs) {
            r.w.offsets(o, oo, oa, ob);
            for (int64_t i = wy; i < r.len; i += 8)
                acc = combine<OP>(acc, transform<OP>(A[oa + i * r.sa_axis],
                                                     OP == ANN_REDUCE_DOT ? Bp[ob + i * r.sb_axis] : T(0)));
        }
        part[wy][lane] = acc;
        __syncthreads();
        if (wy == 0 && o < r.outputs) {
            T v = part[0][lane];
            for (int k = 1; k < 8; ++k) v = combine<OP>(v, part[k][lane]);
            out[oo] = finalize<OP>(v, r.len);
        }
        __syncthreads();
    }
}

// The same 32 adjacent outputs per tile, but a cluster of kColSplit CTAs per
// tile: CTA k of the cluster reduces the k-th slice of the axis (its 8 warps
// interleaved over the slice, four loads in flight per thread) and CTA 0 then
// combines the slices' partials in rank order through distributed shared
// memory. Eight times the CTAs of reduce_cols for the same outputs, which is
// what a long axis with few outputs needs to keep HBM busy; the combine order
// is fixed, so results do not depend on timing.
constexpr int kColSplit = 8;

template <int OP, typename T>
__global__ void __launch_bounds__(kThreads) reduce_cols_cluster(ReduceArgs r) {
    __shared__ T part[8][33];
    __shared__ T cta[32];
    cg::cluster_group cluster = cg::this_cluster();
    int const rank = static_cast<int>(cluster.block_rank());
    T const* A = static_cast<T const*>(r.a);
    T const* Bp = static_cast<T const*>(r.b);
    T* out = static_cast<T*>(r.out);
    int const lane = threadIdx.x & 31, wy = threadIdx.x >> 5;
    int64_t const tiles = ceil_div(r.outputs, 32);
    int64_t const clusters = gridDim.x / kColSplit;
    int64_t const per = ceil_div(r.len, kColSplit);
    int64_t const lo = rank * per < r.len ? rank * per : r.len;
    int64_t const hi = lo + per < r.len ? lo + per : r.len;
    for (int64_t t = blockIdx.x / kColSplit; t < tiles; t += clusters) {  // same trip count in every CTA
        int64_t const o = t * 32 + lane;
        T acc = reduce_init<OP, T>();
        int64_t oo = 0, oa = 0, ob = 0;
        if (o < r.outputs) {
            r.w.offsets(o, oo, oa, ob);
            auto term = [&](int64_t i) {
                return transform<OP>(A[oa + i * r.sa_axis], OP == ANN_REDUCE_DOT ? Bp[ob + i * r.sb_axis] : T(0));
            };
            int64_t i = lo + wy;
            for (; i + 24 < hi; i += 32) {
                T const t0 = term(i), t1 = term(i + 8), t2 = term(i + 16), t3 = term(i + 24);
                acc = combine<OP>(combine<OP>(combine<OP>(combine<OP>(acc, t0), t1), t2), t3);
            }
            for (; i < hi; i += 8) acc = combine<OP>(acc, term(i));
        }
        part[wy][lane] = acc;
        __syncthreads();
        if (wy == 0) {
            T v = part[0][lane];
#pragma unroll
            for (int k = 1; k < 8; ++k) v = combine<OP>(v, part[k][lane]);
            cta[lane] = v;
        }
        cluster.sync();
        if (rank == 0 && wy == 0 && o < r.outputs) {
            T v = cta[lane];
            for (int k = 1; k < kColSplit; ++k) v = combine<OP>(v, cluster.map_shared_rank(cta, k)[lane]);
            out[oo] = finalize<OP>(v, r.len);
        }
        cluster.sync();  // the peers' partials must outlive rank 0's reads
    }
}

template <int OP, typename T>
int launch_cols_cluster(cudaStream_t s, ReduceArgs const& r) {
    int64_t const tiles = ceil_div(r.outputs, 32);
    int64_t clusters = static_cast<int64_t>(sm_count()) * 8 / kColSplit;
    if (clusters > tiles) clusters = tiles;
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = kColSplit;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(clusters * kColSplit));
    cfg.blockDim = dim3(kThreads);
    cfg.stream = s;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    cudaError_t const e = cudaLaunchKernelEx(&cfg, reduce_cols_cluster<OP, T>, r);
    if (e != cudaSuccess) return fail(ANN_ECUDA, "reduce: %s", cudaGetErrorString(e));
    return ANN_OK;
}

char const* reduce_name(int op) {
    switch (op) {
        case ANN_REDUCE_SUM: return "reduceSum";
        case ANN_REDUCE_MAX: return "reduceMax";
        case ANN_REDUCE_MEAN: return "reduceMean";
        case ANN_REDUCE_SUM_SQUARES: return "reduceSumSquares";
        default: return "dot";
    }
}

// The plain column case: the reduced axis is the outermost one and the rest
// is one contiguous run in a, b and out (output o at offset o everywhere),
// 16-byte aligned. A cluster of kColSplit CTAs splits the axis; a CTA owns
// 16 * NV columns, each half-warp one row at a time (16 lanes x 16 bytes),
// four rows in flight a thread, the 16 half-warps' partials then combined
// in order through shared memory and the cluster's in rank order through
// distributed shared memory.
template <int OP, typename T>
__global__ void __launch_bounds__(kThreads) reduce_cols_vec(ReduceArgs r) {
    using V = typename Vec16<T>::type;
    constexpr int NV = Vec16<T>::n, TC = 16 * NV;
    __shared__ T part[16][TC + 1];
    __shared__ T cta[TC];
    cg::cluster_group cluster = cg::this_cluster();
    int const rank = static_cast<int>(cluster.block_rank());
    T const* A = static_cast<T const*>(r.a);
    T const* Bp = static_cast<T const*>(r.b);
    T* out = static_cast<T*>(r.out);
    int const l16 = threadIdx.x & 15, half = threadIdx.x >> 4;
    int64_t const tiles = r.outputs / TC;  // outputs is a multiple of TC here
    int64_t const clusters = gridDim.x / kColSplit;
    int64_t const per = ceil_div(r.len, kColSplit);
    int64_t const lo = rank * per < r.len ? rank * per : r.len;
    int64_t const hi = lo + per < r.len ? lo + per : r.len;
    auto term = [&](V x, V y, T* acc) {
        T const* xe = reinterpret_cast<T const*>(&x);
        T const* ye = reinterpret_cast<T const*>(&y);
#pragma unroll
        for (int k = 0; k < NV; ++k) acc[k] = combine<OP>(acc[k], transform<OP>(xe[k], ye[k]));
    };
    for (int64_t t = blockIdx.x / kColSplit; t < tiles; t += clusters) {  // same trip count in every CTA
        int64_t const c0 = t * TC + l16 * NV;
        T acc[NV];
#pragma unroll
        for (int k = 0; k < NV; ++k) acc[k] = reduce_init<OP, T>();
        int64_t i = lo + half;
        for (; i + 48 < hi; i += 64) {
            V x[4], y[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                x[u] = *reinterpret_cast<V const*>(A + (i + 16 * u) * r.sa_axis + c0);
                y[u] = OP == ANN_REDUCE_DOT ? *reinterpret_cast<V const*>(Bp + (i + 16 * u) * r.sb_axis + c0) : V{};
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) term(x[u], y[u], acc);
        }
        for (; i < hi; i += 16) {
            V const x = *reinterpret_cast<V const*>(A + i * r.sa_axis + c0);
            V const y = OP == ANN_REDUCE_DOT ? *reinterpret_cast<V const*>(Bp + i * r.sb_axis + c0) : V{};
            term(x, y, acc);
        }
#pragma unroll
        for (int k = 0; k < NV; ++k) part[half][l16 * NV + k] = acc[k];
        __syncthreads();
        if (threadIdx.x < TC) {
            T v = part[0][threadIdx.x];
#pragma unroll
            for (int h = 1; h < 16; ++h) v = combine<OP>(v, part[h][threadIdx.x]);
            cta[threadIdx.x] = v;
        }
        cluster.sync();
        if (rank == 0 && threadIdx.x < TC) {
            T v = cta[threadIdx.x];
            for (int k = 1; k < kColSplit; ++k) v = combine<OP>(v, cluster.map_shared_rank(cta, k)[threadIdx.x]);
            out[t * TC + threadIdx.x] = finalize<OP>(v, r.len);
        }
        cluster.sync();  // the peers' partials must outlive rank 0's reads, and part is reused
    }
}

template <int OP, typename T>
int launch_cols_vec(cudaStream_t s, ReduceArgs const& r) {
    constexpr int TC = 16 * Vec16<T>::n;
    int64_t const tiles = r.outputs / TC;
    int64_t clusters = static_cast<int64_t>(sm_count()) * 8 / kColSplit;
    if (clusters > tiles) clusters = tiles;
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = kColSplit;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(clusters * kColSplit));
    cfg.blockDim = dim3(kThreads);
    cfg.stream = s;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    cudaError_t const e = cudaLaunchKernelEx(&cfg, reduce_cols_vec<OP, T>, r);
    if (e != cudaSuccess) return fail(ANN_ECUDA, "reduce: %s", cudaGetErrorString(e));
    return ANN_OK;
}

template <int OP, typename T>
int launch_reduce(cudaStream_t s, ReduceArgs const& r, bool rows, bool vec, bool plain_cols = false) {
    if (!rows && plain_cols) return launch_cols_vec<OP, T>(s, r);
    if (!rows) {
        // few output tiles against a long axis: split the axis over a cluster
        if (r.len >= 256 && ceil_div(r.outputs, 32) < 4 * sm_count()) return launch_cols_cluster<OP, T>(s, r);
        reduce_cols<OP, T><<<grid_for(ceil_div(r.outputs, 32), 1, 8), kThreads, 0, s>>>(r);
    } else if (vec && (r.len <= 65536 || r.outputs >= 4 * sm_count())) {
        reduce_rows_vec<OP, T><<<grid_for(r.outputs, kThreads / 32, 8), kThreads, 0, s>>>(r);
    } else if (r.len <= 2048) {
        reduce_rows<OP, T, 32><<<grid_for(r.outputs, kThreads / 32, 8), kThreads, 0, s>>>(r);
    } else {
        reduce_rows<OP, T, kThreads><<<grid_for(r.outputs, 1, 8), kThreads, 0, s>>>(r);
    }
    return ANN_OK;
}

// validateReduction (reduction.hpp:173-188) and the launch.
template <typename T>
int reduce(ann_stream stream, int op, const ann_view* a_v, const ann_view* b_v, const ann_view* out_v,
           uint32_t axis) {
    char const* name = reduce_name(op);
    if (op < ANN_REDUCE_SUM || op > ANN_REDUCE_DOT) return fail(ANN_EINVAL, "reduce: unknown operator %d.", op);
    Dims a, b, out;
    ANN_TRY(to_dims(a_v, sizeof(T), name, a));
    ANN_TRY(to_dims(out_v, sizeof(T), name, out));
    if (a.rank != out.rank) return fail(ANN_EINVAL, "%s requires output rank to match input rank.", name);
    if (axis >= static_cast<uint32_t>(a.rank)) return fail(ANN_EINVAL, "%s axis out of range.", name);
    for (int i = 0; i < a.rank; ++i)
        if (out.ext[i] != (i == static_cast<int>(axis) ? 1 : a.ext[i]))
            return fail(ANN_EINVAL, "%s output extents mismatch.", name);
    if (op == ANN_REDUCE_DOT) {
        ANN_TRY(to_dims(b_v, sizeof(T), name, b));
        if (!same_extents(a, b)) return fail(ANN_EINVAL, "dot shape mismatch.");
    }
    if (out.numel() == 0) return ANN_OK;
    ReduceArgs r{};
    r.a = a.data;
    r.b = op == ANN_REDUCE_DOT ? b.data : a.data;
    r.out = out.data;
    r.len = a.ext[axis];
    r.outputs = out.numel();
    r.sa_axis = a.str[axis];
    r.sb_axis = op == ANN_REDUCE_DOT ? b.str[axis] : a.str[axis];
    r.w = walk_of(out, &out, &a, op == ANN_REDUCE_DOT ? &b : &a);
    bool const rows = r.sa_axis == 1 && r.sb_axis == 1 && r.len >= 16;
    // 16-byte vectors need every row start aligned: the base pointers and
    // every non-reduced stride a multiple of the vector width.
    bool vec = rows && aligned(a.data, 16) && (op != ANN_REDUCE_DOT || aligned(b.data, 16));
    for (int i = 0; vec && i < a.rank; ++i) {
        if (i == static_cast<int>(axis) || a.ext[i] == 1) continue;
        vec = a.str[i] % Vec16<T>::n == 0 && (op != ANN_REDUCE_DOT || b.str[i] % Vec16<T>::n == 0);
    }
    // The plain column case for reduce_cols_vec: every non-reduced axis of
    // extent > 1 row-major contiguous, innermost first, in a, b and out, the
    // reduced axis outermost of them, 16-byte aligned rows, the outputs a
    // whole number of column tiles and an axis long enough to split.
    bool plain = !rows && r.len >= 256;
    {
        int64_t expect = 1;
        for (int i = a.rank - 1; plain && i >= 0; --i) {
            if (i == static_cast<int>(axis) || a.ext[i] == 1) continue;
            plain = a.str[i] == expect && out.str[i] == expect && (op != ANN_REDUCE_DOT || b.str[i] == expect) &&
                    static_cast<int>(axis) < i;
            expect *= a.ext[i];
        }
        constexpr int NV = Vec16<T>::n;
        plain = plain && r.outputs % (16 * NV) == 0 && r.sa_axis % NV == 0 && r.sb_axis % NV == 0 &&
                aligned(a.data, 16) && aligned(out.data, 16) && (op != ANN_REDUCE_DOT || aligned(b.data, 16));
    }
    cudaStream_t s = as_stream(stream);
    switch (op) {
        case ANN_REDUCE_SUM: ANN_TRY((launch_reduce<ANN_REDUCE_SUM, T>(s, r, rows, vec, plain))); break;
        case ANN_REDUCE_MAX: ANN_TRY((launch_reduce<ANN_REDUCE_MAX, T>(s, r, rows, vec, plain))); break;
        case ANN_REDUCE_MEAN: ANN_TRY((launch_reduce<ANN_REDUCE_MEAN, T>(s, r, rows, vec, plain))); break;
        case ANN_REDUCE_SUM_SQUARES:
            ANN_TRY((launch_reduce<ANN_REDUCE_SUM_SQUARES, T>(s, r, rows, vec, plain)));
            break;
        default: ANN_TRY((launch_reduce<ANN_REDUCE_DOT, T>(s, r, rows, vec, plain))); break;
    }
    return check_launch(name);
}

}  // namespace
}  // namespace ann

extern "C" {

int ann_unary_f32(ann_stream s, int32_t op, const ann_view* in, const ann_view* out, float scalar) {
    ANN_API_BEGIN
    return ann::unary_op<float>(s, op, in, out, scalar);
    ANN_API_END
}
int ann_unary_f64(ann_stream s, int32_t op, const ann_view* in, const ann_view* out, double scalar) {
    ANN_API_BEGIN
    return ann::unary_op<double>(s, op, in, out, scalar);
    ANN_API_END
}
int ann_binary_f32(ann_stream s, int32_t op, const ann_view* lhs, const ann_view* rhs, const ann_view* out,
                   float alpha) {
    ANN_API_BEGIN
    return ann::binary_op<float>(s, op, lhs, rhs, out, alpha);
    ANN_API_END
}
int ann_binary_f64(ann_stream s, int32_t op, const ann_view* lhs, const ann_view* rhs, const ann_view* out,
                   double alpha) {
    ANN_API_BEGIN
    return ann::binary_op<double>(s, op, lhs, rhs, out, alpha);
    ANN_API_END
}
int ann_bias_add_f32(ann_stream s, const ann_view* in, const ann_view* bias, int32_t act, const ann_view* out) {
    ANN_API_BEGIN
    return ann::bias_act<float>(s, in, bias, act, out);
    ANN_API_END
}
int ann_bias_add_f64(ann_stream s, const ann_view* in, const ann_view* bias, int32_t act, const ann_view* out) {
    ANN_API_BEGIN
    return ann::bias_act<double>(s, in, bias, act, out);
    ANN_API_END
}

int ann_cast(ann_stream stream, const ann_view* in_v, int32_t in_dtype, const ann_view* out_v, int32_t out_dtype) {
    ANN_API_BEGIN
    size_t const isz = ann::dtype_size(in_dtype), osz = ann::dtype_size(out_dtype);
    if (!isz || !osz) return ann::fail(ANN_EINVAL, "cast: unknown element type.");
    ann::Dims in, out;
    ANN_TRY(ann::to_dims(in_v, isz, "cast input", in));
    ANN_TRY(ann::to_dims(out_v, osz, "cast output", out));
    if (!ann::same_extents(in, out)) return ann::fail(ANN_EINVAL, "cast shape mismatch.");
    if (out.numel() == 0) return ANN_OK;
    cudaStream_t s = ann::as_stream(stream);
    int const dense = in.dense() && out.dense();
    switch (out_dtype) {
        case ANN_DTYPE_F32: ann::cast_from<float>(s, in_dtype, in, out, dense); break;
        case ANN_DTYPE_F64: ann::cast_from<double>(s, in_dtype, in, out, dense); break;
        case ANN_DTYPE_I32: ann::cast_from<int32_t>(s, in_dtype, in, out, dense); break;
        case ANN_DTYPE_U32: ann::cast_from<uint32_t>(s, in_dtype, in, out, dense); break;
        default: ann::cast_from<int64_t>(s, in_dtype, in, out, dense); break;
    }
    return ann::check_launch("cast");
    ANN_API_END
}

int ann_fill(ann_stream stream, const ann_view* out_v, int32_t dtype, const void* value) {
    ANN_API_BEGIN
    size_t const sz = ann::dtype_size(dtype);
    if (!sz) return ann::fail(ANN_EINVAL, "fill: unknown element type.");
    if (!value) return ann::fail(ANN_EINVAL, "fill: value is NULL.");
    ann::Dims out;
    ANN_TRY(ann::to_dims(out_v, sz, "fill output", out));
    if (out.numel() == 0) return ANN_OK;
    cudaStream_t s = ann::as_stream(stream);
    switch (dtype) {
        case ANN_DTYPE_F32: ann::fill_as<float>(s, out, value); break;
        case ANN_DTYPE_F64: ann::fill_as<double>(s, out, value); break;
        case ANN_DTYPE_I32: ann::fill_as<int32_t>(s, out, value); break;
        case ANN_DTYPE_U32: ann::fill_as<uint32_t>(s, out, value); break;
        default: ann::fill_as<int64_t>(s, out, value); break;
    }
    return ann::check_launch("fill");
    ANN_API_END
}

int ann_reduce_f32(ann_stream s, int32_t op, const ann_view* in, const ann_view* out, uint32_t axis) {
    ANN_API_BEGIN
    if (op == ANN_REDUCE_DOT) return ann::fail(ANN_EINVAL, "reduce: use ann_dot_f32 for dot.");
    return ann::reduce<float>(s, op, in, nullptr, out, axis);
    ANN_API_END
}
int ann_reduce_f64(ann_stream s, int32_t op, const ann_view* in, const ann_view* out, uint32_t axis) {
    ANN_API_BEGIN
    if (op == ANN_REDUCE_DOT) return ann::fail(ANN_EINVAL, "reduce: use ann_dot_f64 for dot.");
    return ann::reduce<double>(s, op, in, nullptr, out, axis);
    ANN_API_END
}
int ann_dot_f32(ann_stream s, const ann_view* lhs, const ann_view* rhs, const ann_view* out, uint32_t axis) {
    ANN_API_BEGIN
    return ann::reduce<float>(s, ANN_REDUCE_DOT, lhs, rhs, out, axis);
    ANN_API_END
}
int ann_dot_f64(ann_stream s, const ann_view* lhs, const ann_view* rhs, const ann_view* out, uint32_t axis) {
    ANN_API_BEGIN
    return ann::reduce<double>(s, ANN_REDUCE_DOT, lhs, rhs, out, axis);
    ANN_API_END
}

}  // extern "C"
