// rms_norm.cu -- rmsNorm (reference: onHost/nn/rms_norm.hpp:17-35,
// onAcc/internal/nn/rms_norm.hpp:19-39): y = x * rsqrt(sum(x^2)/H + eps) * w
// along the last axis.
//
// The reference recomputes the row sum once per OUTPUT element (O(N*H^2));
// here a row is reduced once by a warp (H <= 1024) or a whole 256-thread CTA
// (longer rows) with 16-byte loads, then scaled on a second, cache-hot pass:
// one HBM read and one HBM write per element. The multiplication order
// x * rms * w of the reference is kept.
#include "common.cuh"
#include "reduce.cuh"

namespace ann {
namespace {

struct RmsArgs {
    const void* in;
    void* out;
    const void* w;
    int64_t rows, hidden, s_in, s_out, s_w;
    Outer2 outer;
};

template <typename T, int GROUP, bool VEC>
__global__ void __launch_bounds__(256) rms_norm_kernel(RmsArgs a, T eps) {
    using V = typename Vec16<T>::type;
    constexpr int NV = Vec16<T>::n;
    constexpr int RPB = 256 / GROUP;  // rows per block per iteration
    __shared__ T scratch[8];
    int const gl = threadIdx.x % GROUP;
    T const* in = static_cast<T const*>(a.in);
    T const* w = static_cast<T const*>(a.w);
    T* out = static_cast<T*>(a.out);
    int64_t const iters = ceil_div(a.rows, static_cast<int64_t>(gridDim.x) * RPB);
    for (int64_t it = 0; it < iters; ++it) {
        int64_t const row = (it * gridDim.x + blockIdx.x) * RPB + threadIdx.x / GROUP;
        bool const live = row < a.rows;
        int64_t oi = 0, oo = 0;
        if (live) a.outer.offsets(row, oi, oo);
        T sum{};
        if (live) {
            if constexpr (VEC) {
                V const* x = reinterpret_cast<V const*>(in + oi);
                for (int64_t v = gl; v < a.hidden / NV; v += GROUP) {
                    V const xv = x[v];
                    if constexpr (NV == 4) {
                        sum += xv.x * xv.x; sum += xv.y * xv.y; sum += xv.z * xv.z; sum += xv.w * xv.w;
                    } else {
                        sum += xv.x * xv.x; sum += xv.y * xv.y;
                    }
                }
            } else {
                for (int64_t h = gl; h < a.hidden; h += GROUP) {
                    T const x = in[oi + h * a.s_in];
                    sum += x * x;
                }
            }
        }
        if constexpr (GROUP == 32) {
            sum = warp_sum(sum);
        } else {
            sum = block_sum<8>(sum, scratch);
        }
        if (!live) continue;
        T const rms = rsqrt_t(sum / static_cast<T>(a.hidden) + eps);
        if constexpr (VEC) {
            V const* x = reinterpret_cast<V const*>(in + oi);
            V const* wv = reinterpret_cast<V const*>(w);
            V* y = reinterpret_cast<V*>(out + oo);
            for (int64_t v = gl; v < a.hidden / NV; v += GROUP) {
                V const xv = x[v];
                V const ww = __ldg(wv + v);
                V r;
                if constexpr (NV == 4) {
                    r.x = xv.x * rms * ww.x; r.y = xv.y * rms * ww.y; r.z = xv.z * rms * ww.z; r.w = xv.w * rms * ww.w;
                } else {
                    r.x = xv.x * rms * ww.x; r.y = xv.y * rms * ww.y;
                }
                y[v] = r;
            }
        } else {
            for (int64_t h = gl; h < a.hidden; h += GROUP)
                out[oo + h * a.s_out] = in[oi + h * a.s_in] * rms * w[h * a.s_w];
        }
    }
}

template <typename T>
int rms_norm(ann_stream stream, const ann_view* in_v, const ann_view* w_v, const ann_view* out_v, T eps) {
    Dims in, w, out;
    ANN_TRY(to_dims(in_v, sizeof(T), "rmsNorm input", in));
    ANN_TRY(to_dims(w_v, sizeof(T), "rmsNorm weight", w));
    ANN_TRY(to_dims(out_v, sizeof(T), "rmsNorm output", out));
    // rms_norm.hpp:21-25
    if (!same_extents(in, out)) return fail(ANN_EINVAL, "rmsNorm shape mismatch.");
    if (w.rank != 1 || w.ext[0] != in.ext[in.rank - 1])
        return fail(ANN_EINVAL, "rmsNorm expects a 1D weight matching the last axis.");
    if (in.numel() == 0) return ANN_OK;

    RmsArgs a{};
    a.in = in.data;
    a.out = out.data;
    a.w = w.data;
    a.hidden = in.ext[in.rank - 1];
    a.rows = in.numel() / a.hidden;
    a.s_in = in.str[in.rank - 1];
    a.s_out = out.str[out.rank - 1];
    a.s_w = w.str[0];
    a.outer.n = in.rank - 1;
    bool outer_aligned = true;
    for (int i = 0; i < in.rank - 1; ++i) {
        a.outer.ext[i] = in.ext[i];
        a.outer.sa[i] = in.str[i];
        a.outer.sb[i] = out.str[i];
        outer_aligned = outer_aligned && (in.str[i] * sizeof(T)) % 16 == 0 && (out.str[i] * sizeof(T)) % 16 == 0;
    }
    constexpr int NV = Vec16<T>::n;
    bool const vec = a.s_in == 1 && a.s_out == 1 && a.s_w == 1 && a.hidden % NV == 0 && outer_aligned &&
                     aligned(in.data, 16) && aligned(out.data, 16) && aligned(w.data, 16);
    cudaStream_t s = as_stream(stream);
    if (a.hidden <= 1024) {
        int const grid = grid_for(a.rows, 8);
        if (vec) rms_norm_kernel<T, 32, true><<<grid, 256, 0, s>>>(a, eps);
        else rms_norm_kernel<T, 32, false><<<grid, 256, 0, s>>>(a, eps);
    } else {
        int const grid = grid_for(a.rows, 1, 8);
        if (vec) rms_norm_kernel<T, 256, true><<<grid, 256, 0, s>>>(a, eps);
        else rms_norm_kernel<T, 256, false><<<grid, 256, 0, s>>>(a, eps);
    }
    return check_launch("rmsNorm");
}

}  // namespace
}  // namespace ann

extern "C" {

int ann_rms_norm_f32(ann_stream s, const ann_view* in, const ann_view* w, const ann_view* out, float eps) {
    ANN_API_BEGIN
    return ann::rms_norm<float>(s, in, w, out, eps);
    ANN_API_END
}

int ann_rms_norm_f64(ann_stream s, const ann_view* in, const ann_view* w, const ann_view* out, double eps) {
    ANN_API_BEGIN
    return ann::rms_norm<double>(s, in, w, out, eps);
    ANN_API_END
}

}  // extern "C"
