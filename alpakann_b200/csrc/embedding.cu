// embedding.cu -- embeddingLookup (reference: onHost/nn/embedding.hpp:17-36,
// onAcc/internal/nn/embedding.hpp:15-24): out[t, :] = table[ids[t], :].
//
// B200 shape: one warp per output row, 16-byte vector copies when both rows
// are contiguous and aligned (a row gather is pure HBM traffic), strided
// element copies otherwise (non-contiguous subviews, as in the reference's
// subview test). A copy, so bit-exact by construction.
#include "common.cuh"

namespace ann {
namespace {

__device__ unsigned int g_device_error;  // ANN_DEVERR_* bits, read by ann_take_device_error

struct EmbedArgs {
    const uint32_t* ids;
    int64_t ids_stride;
    const void* table;
    int64_t vocab, tab_row, tab_col;
    void* out;
    int64_t out_row, out_col;
    int64_t rows, hidden;
};

template <typename T, bool VEC>
__global__ void __launch_bounds__(256) embedding_kernel(EmbedArgs a) {
    using V = typename Vec16<T>::type;
    constexpr int NV = Vec16<T>::n;
    int const lane = threadIdx.x & 31;
    int64_t const warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    T const* table = static_cast<T const*>(a.table);
    T* out = static_cast<T*>(a.out);
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < a.rows;
         t += warps) {
        uint32_t const id = __ldg(a.ids + t * a.ids_stride);
        T* dst = out + t * a.out_row;
        if (static_cast<int64_t>(id) >= a.vocab) {
            // The reference reads out of bounds here; write a zero row and flag it.
            for (int64_t h = lane; h < a.hidden; h += 32) dst[h * a.out_col] = T{};
            if (lane == 0) atomicOr(&g_device_error, ANN_DEVERR_TOKEN_ID);
            continue;
        }
        T const* src = table + static_cast<int64_t>(id) * a.tab_row;
        if constexpr (VEC) {
            V const* s = reinterpret_cast<V const*>(src);
            V* d = reinterpret_cast<V*>(dst);
            int64_t const nv = a.hidden / NV;
            for (int64_t h = lane; h < nv; h += 32) d[h] = __ldg(s + h);
        } else {
            for (int64_t h = lane; h < a.hidden; h += 32) dst[h * a.out_col] = src[h * a.tab_col];
        }
    }
}

template <typename T>
int embedding_lookup(ann_stream stream, const ann_view* ids_v, const ann_view* table_v, const ann_view* out_v) {
    Dims ids, table, out;
    ANN_TRY(to_dims(ids_v, sizeof(uint32_t), "embeddingLookup ids", ids));
    ANN_TRY(to_dims(table_v, sizeof(T), "embeddingLookup embedding", table));
    ANN_TRY(to_dims(out_v, sizeof(T), "embeddingLookup output", out));
    // embedding.hpp:23-27
    if (ids.rank != 1 || table.rank != 2 || out.rank != 2)
        return fail(ANN_EINVAL, "embeddingLookup expects 1D ids and 2D embedding/output.");
    if (out.ext[0] != ids.ext[0] || out.ext[1] != table.ext[1])
        return fail(ANN_EINVAL, "embeddingLookup shape mismatch.");
    if (out.numel() == 0) return ANN_OK;

    EmbedArgs a{static_cast<const uint32_t*>(ids.data), ids.str[0], table.data, table.ext[0], table.str[0],
                table.str[1], out.data, out.str[0], out.str[1], out.ext[0], out.ext[1]};
    constexpr int NV = Vec16<T>::n;
    bool const vec = table.str[1] == 1 && out.str[1] == 1 && a.hidden % NV == 0 && aligned(table.data, 16) &&
                     aligned(out.data, 16) && (table.str[0] * sizeof(T)) % 16 == 0 &&
                     (out.str[0] * sizeof(T)) % 16 == 0;
    int const grid = grid_for(a.rows, 8);
    if (vec)
        embedding_kernel<T, true><<<grid, 256, 0, as_stream(stream)>>>(a);
    else
        embedding_kernel<T, false><<<grid, 256, 0, as_stream(stream)>>>(a);
    return check_launch("embeddingLookup");
}

}  // namespace

int take_embedding_error(cudaStream_t s, uint32_t* bits) {
    unsigned int value = 0, zero = 0;
    if (cudaMemcpyFromSymbolAsync(&value, g_device_error, sizeof value, 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ANN_ECUDA, "device error word: %s", cudaGetErrorString(cudaGetLastError()));
    *bits |= value;
    return ANN_OK;
}

}  // namespace ann

extern "C" {

int ann_embedding_lookup_f32(ann_stream s, const ann_view* ids, const ann_view* table, const ann_view* out) {
    ANN_API_BEGIN
    return ann::embedding_lookup<float>(s, ids, table, out);
    ANN_API_END
}

int ann_embedding_lookup_f64(ann_stream s, const ann_view* ids, const ann_view* table, const ann_view* out) {
    ANN_API_BEGIN
    return ann::embedding_lookup<double>(s, ids, table, out);
    ANN_API_END
}

}  // extern "C"
