// rms_norm.cu -- rmsNorm (reference: onHost/nn/rms_norm.hpp:17-35,
// onAcc/internal/nn/rms_norm.hpp:19-39): y = x * rsqrt(sum(x^2)/H + eps) * w
// along the last axis.
//
// The reference recomputes the row sum once per OUTPUT element (O(N*H^2));
// here a row is reduced once by a warp (H <= 1024) or a whole 256-thread CTA
// (longer rows) with 16-byte loads, then scaled on a second, cache-hot pass:
// one HBM read and one HBM write per element. The multiplication order
// x * rms * w of the reference is kept.
//
// embeddingRmsNorm fuses the path's first two steps, embeddingLookup
// (onAcc/internal/nn/embedding.hpp:15-24) and rmsNorm: row r is read straight
// from embedding[ids[r]] by the same kernel, so the result is bit for bit the
// two-launch result without the hidden state's round trip through HBM.
#include "common.cuh"
#include "reduce.cuh"

namespace ann {

int take_rms_error(cudaStream_t s, uint32_t* bits);

namespace {

__device__ unsigned int g_rms_error;  // ANN_DEVERR_TOKEN_ID from embeddingRmsNorm

struct RmsArgs {
    const void* in;  // input rows, or the embedding table when gathering
    void* out;
    const void* w;
    int64_t rows, hidden, s_in, s_out, s_w;
    Outer2 outer;
    // gather: row r is embedding row ids[r * s_ids] (pitch s_row) if < vocab
    const uint32_t* ids;
    int64_t s_ids, s_row, vocab;
};

// Aligned rows of at most GROUP * CH 16-byte vectors: the row is held in
// registers, CH vectors a thread (v = gl + GROUP c), all loads issued before
// the first is used, and the second pass reads the registers instead of the
// row again. The squares are summed in the same order as rms_norm_kernel's
// loop (the extra terms are +0), so both give the same bits.
template <typename T, int GROUP, int CH, bool GATHER>
__global__ void __launch_bounds__(256) rms_norm_regs(RmsArgs a, T eps) {
    using V = typename Vec16<T>::type;
    constexpr int NV = Vec16<T>::n;
    constexpr int RPB = 256 / GROUP;
    __shared__ T scratch[8];
    int const gl = threadIdx.x % GROUP;
    T const* in = static_cast<T const*>(a.in);
    V const* wv = static_cast<V const*>(a.w);
    T* out = static_cast<T*>(a.out);
    int const nvec = static_cast<int>(a.hidden / NV);  // <= GROUP * CH
    int64_t const iters = ceil_div(a.rows, static_cast<int64_t>(gridDim.x) * RPB);
    for (int64_t it = 0; it < iters; ++it) {
        int64_t const row = (it * gridDim.x + blockIdx.x) * RPB + threadIdx.x / GROUP;
        bool const live = row < a.rows;
        bool valid = live;
        int64_t oi = 0, oo = 0;
        if (live) {
            a.outer.offsets(row, oi, oo);
            if constexpr (GATHER) {
                uint32_t const id = a.ids[row * a.s_ids];
                valid = id < a.vocab;
                if (!valid && gl == 0) atomicOr(&g_rms_error, ANN_DEVERR_TOKEN_ID);
                oi = static_cast<int64_t>(id) * a.s_row;
            }
        }
        V const* x = reinterpret_cast<V const*>(in + oi);
        V xr[CH];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            int const v = gl + GROUP * c;
            xr[c] = (valid && v < nvec) ? x[v] : V{};
        }
        T sum{};
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            V const xv = xr[c];
            if constexpr (NV == 4) {
                sum += xv.x * xv.x; sum += xv.y * xv.y; sum += xv.z * xv.z; sum += xv.w * xv.w;
            } else {
                sum += xv.x * xv.x; sum += xv.y * xv.y;
            }
        }
        if constexpr (GROUP == 32) {
            sum = warp_sum(sum);
        } else {
            sum = block_sum<8>(sum, scratch);
        }
        if (!live) continue;
        T const rms = rsqrt_t(sum / static_cast<T>(a.hidden) + eps);
        V* y = reinterpret_cast<V*>(out + oo);
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            int const v = gl + GROUP * c;
            if (v >= nvec) continue;
            V r{};
            if (valid) {  // an id out of range gives a zero row, as embeddingLookup writes
                V const xv = xr[c];
                V const ww = __ldg(wv + v);
                if constexpr (NV == 4) {
                    r.x = xv.x * rms * ww.x; r.y = xv.y * rms * ww.y; r.z = xv.z * rms * ww.z; r.w = xv.w * rms * ww.w;
                } else {
                    r.x = xv.x * rms * ww.x; r.y = xv.y * rms * ww.y;
                }
            }
            y[v] = r;
        }
    }
}

template <typename T, int GROUP, bool VEC, bool GATHER>
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
        bool live = row < a.rows;
        bool valid = live;  // false: a gathered id out of range -> a zero row, as embeddingLookup writes
        int64_t oi = 0, oo = 0;
        if (live) {
            a.outer.offsets(row, oi, oo);
            if constexpr (GATHER) {
                uint32_t const id = a.ids[row * a.s_ids];
                valid = id < a.vocab;
                if (!valid && gl == 0) atomicOr(&g_rms_error, ANN_DEVERR_TOKEN_ID);
                oi = static_cast<int64_t>(id) * a.s_row;
            }
        }
        T sum{};
        if (valid) {
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
        if (!valid) {
            for (int64_t h = gl; h < a.hidden; h += GROUP) out[oo + h * a.s_out] = T{};
            continue;
        }
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

template <typename T, bool GATHER>
int launch_rms(ann_stream stream, RmsArgs const& a, bool vec, T eps, const char* what);

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
    return launch_rms<T, false>(stream, a, vec, eps, "rmsNorm");
}

// One launch with the block shape rmsNorm picks for this row length, so the
// gathered variant reduces in exactly the same order.
template <typename T, bool GATHER>
int launch_rms(ann_stream stream, RmsArgs const& a, bool vec, T eps, const char* what) {
    cudaStream_t s = as_stream(stream);
    constexpr int NV = Vec16<T>::n;
    if (a.hidden <= 1024) {
        int const grid = grid_for(a.rows, 8);
        if (vec && a.hidden <= 32 * 8 * NV) rms_norm_regs<T, 32, 8, GATHER><<<grid, 256, 0, s>>>(a, eps);
        else if (vec) rms_norm_kernel<T, 32, true, GATHER><<<grid, 256, 0, s>>>(a, eps);
        else rms_norm_kernel<T, 32, false, GATHER><<<grid, 256, 0, s>>>(a, eps);
    } else {
        int const grid = grid_for(a.rows, 1, 8);
        if (vec && a.hidden <= 256 * 8 * NV) rms_norm_regs<T, 256, 8, GATHER><<<grid, 256, 0, s>>>(a, eps);
        else if (vec) rms_norm_kernel<T, 256, true, GATHER><<<grid, 256, 0, s>>>(a, eps);
        else rms_norm_kernel<T, 256, false, GATHER><<<grid, 256, 0, s>>>(a, eps);
    }
    return check_launch(what);
}

template <typename T>
int embedding_rms_norm(ann_stream stream, const ann_view* ids_v, const ann_view* table_v, const ann_view* w_v,
                       const ann_view* out_v, T eps) {
    Dims ids, table, w, out;
    ANN_TRY(to_dims(ids_v, sizeof(uint32_t), "embeddingRmsNorm ids", ids));
    ANN_TRY(to_dims(table_v, sizeof(T), "embeddingRmsNorm embedding", table));
    ANN_TRY(to_dims(w_v, sizeof(T), "embeddingRmsNorm weight", w));
    ANN_TRY(to_dims(out_v, sizeof(T), "embeddingRmsNorm output", out));
    // the checks of embeddingLookup (embedding.hpp:23-27) and rmsNorm (rms_norm.hpp:21-25)
    if (ids.rank != 1 || table.rank != 2 || out.rank != 2)
        return fail(ANN_EINVAL, "embeddingLookup expects rank-1 token ids and rank-2 embedding/output.");
    if (out.ext[0] != ids.ext[0] || out.ext[1] != table.ext[1])
        return fail(ANN_EINVAL, "embeddingLookup output shape mismatch.");
    if (w.rank != 1 || w.ext[0] != table.ext[1])
        return fail(ANN_EINVAL, "rmsNorm expects a 1D weight matching the last axis.");
    if (out.numel() == 0) return ANN_OK;
    RmsArgs a{};
    a.in = table.data;
    a.out = out.data;
    a.w = w.data;
    a.hidden = table.ext[1];
    a.rows = ids.ext[0];
    a.s_in = table.str[1];
    a.s_out = out.str[1];
    a.s_w = w.str[0];
    a.outer.n = 1;
    a.outer.ext[0] = a.rows;
    a.outer.sa[0] = 0;  // the input row comes from the id
    a.outer.sb[0] = out.str[0];
    a.ids = static_cast<const uint32_t*>(ids.data);
    a.s_ids = ids.str[0];
    a.s_row = table.str[0];
    a.vocab = table.ext[0];
    constexpr int NV = Vec16<T>::n;
    bool const vec = a.s_in == 1 && a.s_out == 1 && a.s_w == 1 && a.hidden % NV == 0 &&
                     (table.str[0] * sizeof(T)) % 16 == 0 && (out.str[0] * sizeof(T)) % 16 == 0 &&
                     aligned(table.data, 16) && aligned(out.data, 16) && aligned(w.data, 16);
    return launch_rms<T, true>(stream, a, vec, eps, "embeddingRmsNorm");
}

}  // namespace

int take_rms_error(cudaStream_t s, uint32_t* bits) {
    unsigned int value = 0, zero = 0;
    if (cudaMemcpyFromSymbolAsync(&value, g_rms_error, sizeof value, 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_rms_error, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ANN_ECUDA, "device error word: %s", cudaGetErrorString(cudaGetLastError()));
    *bits |= value;
    return ANN_OK;
}

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

int ann_embedding_rms_norm_f32(ann_stream s, const ann_view* ids, const ann_view* embedding, const ann_view* w,
                               const ann_view* out, float eps) {
    ANN_API_BEGIN
    return ann::embedding_rms_norm<float>(s, ids, embedding, w, out, eps);
    ANN_API_END
}

int ann_embedding_rms_norm_f64(ann_stream s, const ann_view* ids, const ann_view* embedding, const ann_view* w,
                               const ann_view* out, double eps) {
    ANN_API_BEGIN
    return ann::embedding_rms_norm<double>(s, ids, embedding, w, out, eps);
    ANN_API_END
}

}  // extern "C"
