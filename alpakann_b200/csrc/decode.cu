// decode.cu -- fused decode attention over a KV cache, split-K.
//
// Computes in ONE launch what the reference's decode pipeline computes in four
// (test/unit/nn/attention.cpp:675-734):
//   attentionScores (onAcc/internal/nn/attention.hpp:21-39)
//   -> ops::scale (onHost/ops/elementwise.hpp:64-73)
//   -> softmax over all keys (onAcc/internal/nn/softmax.hpp:32-74, non-causal)
//   -> attentionApply (onAcc/internal/nn/attention.hpp:49-67)
// without writing the [B,Hq,Tq,Tk] score and probability tensors to memory.
//
// The work is memory-bound (each K/V byte is used for one FMA), so the design
// is about streaming the cache at HBM rate:
//  * grid = query rows x key splits; each CTA owns a contiguous key range of
//    one (batch, query token, query head) row and its KV head (GQA: hq / g);
//  * K and V rows of the range are streamed through a 4-stage ring of 16 KB
//    shared-memory tiles by 1-D bulk copies (TMA, cp.async.bulk) completing on
//    mbarriers: K tiles first (scores), then V tiles (weighted sum), so the V
//    loads are already in flight while the split's softmax is computed;
//  * scores: 8 lanes per key, each lane a 16-byte slice, reduced with three
//    shuffles (conflict-free 128-byte shared-memory phases);
//  * the split's scores stay in shared memory: max, exp and sum are exact
//    over the split, no online rescaling;
//  * splits are merged by the last CTA of a row to finish (completion counter
//    in the workspace) with the log-sum-exp rule
//      out = sum_s e^(m_s - M) acc_s / sum_s e^(m_s - M) l_s.
// Summation order differs from the reference's sequential loops (tree
// reductions, split merge); results agree within the fp32/fp64 tolerances.
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "reduce.cuh"
#include "tma.cuh"

namespace ann {
namespace {

__device__ unsigned int g_decode_error;

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 4;
constexpr int kStageBytes = 16384;
constexpr int kMaxSplits = 64;
constexpr int kMaxChunk = 2048;  // keys per split (scores kept in shared memory)

struct DecodeArgs {
    const void* q;
    const void* k;
    const void* v;
    void* out;
    int64_t q_b, q_t, q_h;        // element strides of Q (unit stride along d)
    int64_t o_b, o_t, o_h, o_d;   // element strides of out
    int64_t k_b, k_h, k_t;        // element strides of K by batch, kv head, token
    int64_t v_b, v_h, v_t;
    int64_t Tq, Hq, Tk, chunk, rows;
    uint32_t g;
    int splits;
    void* part_acc;       // [rows][splits][D]
    void* part_ml;        // [rows][splits][2]
    unsigned int* count;  // [rows]
};

template <typename T, int D>
struct Cfg {
    using V = typename Vec16<T>::type;
    static constexpr int NV = Vec16<T>::n;
    static constexpr int ROWB = D * static_cast<int>(sizeof(T));  // bytes per key row
    static constexpr int VPR = ROWB / 16;                         // 16-byte vectors per row
    static constexpr int TILE = kStageBytes / ROWB;               // keys per stage
    static constexpr int LPK = 8;                                 // score phase: lanes per key
    static constexpr int KPW = 32 / LPK;                          // keys per warp step
    static constexpr int VPL = VPR / LPK;                         // vectors per lane per key
    static constexpr int KPS = VPR >= 32 ? 1 : 32 / VPR;          // PV phase: keys per warp step
    static constexpr int VPLN = VPR >= 32 ? VPR / 32 : 1;         // PV phase: vectors per lane
    static constexpr size_t SMEM = kStages * kStageBytes + kMaxChunk * sizeof(T) + kStages * sizeof(uint64_t);
    static_assert(ROWB % 128 == 0, "row must be a multiple of 128 bytes");
    static_assert(kWarps * D * sizeof(T) <= kStages * kStageBytes, "reduction buffer aliases the stages");
};

template <typename T>
__device__ __forceinline__ T dot16(typename Vec16<T>::type a, typename Vec16<T>::type b, T acc);
template <>
__device__ __forceinline__ float dot16<float>(float4 a, float4 b, float acc) {
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
    acc = fmaf(a.z, b.z, acc);
    return fmaf(a.w, b.w, acc);
}
template <>
__device__ __forceinline__ double dot16<double>(double2 a, double2 b, double acc) {
    acc = fma(a.x, b.x, acc);
    return fma(a.y, b.y, acc);
}

template <typename T>
__device__ __forceinline__ void axpy16(typename Vec16<T>::type& acc, T p, typename Vec16<T>::type v);
template <>
__device__ __forceinline__ void axpy16<float>(float4& acc, float p, float4 v) {
    acc.x = fmaf(p, v.x, acc.x);
    acc.y = fmaf(p, v.y, acc.y);
    acc.z = fmaf(p, v.z, acc.z);
    acc.w = fmaf(p, v.w, acc.w);
}
template <>
__device__ __forceinline__ void axpy16<double>(double2& acc, double p, double2 v) {
    acc.x = fma(p, v.x, acc.x);
    acc.y = fma(p, v.y, acc.y);
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) decode_kernel(DecodeArgs a, T scale) {
    using C = Cfg<T, D>;
    using V = typename C::V;
    extern __shared__ __align__(128) unsigned char smem[];
    T* sc = reinterpret_cast<T*>(smem + kStages * kStageBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes + kMaxChunk * sizeof(T));
    __shared__ T red_s[kWarps];
    __shared__ int s_last;

    int const tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int64_t const bid = blockIdx.x;
    int const split = static_cast<int>(bid % a.splits);
    int64_t const row = bid / a.splits;
    int64_t const hq = row % a.Hq;
    int64_t const tq = (row / a.Hq) % a.Tq;
    int64_t const b = row / (a.Hq * a.Tq);
    int64_t const kvh = hq / a.g;
    int64_t const key0 = static_cast<int64_t>(split) * a.chunk;
    int64_t const left = a.Tk - key0;
    int const nkeys = static_cast<int>(left <= 0 ? 0 : (left < a.chunk ? left : a.chunk));
    int const ntile = (nkeys + C::TILE - 1) / C::TILE;
    int const total = 2 * ntile;

    T const* kbase = static_cast<T const*>(a.k) + b * a.k_b + kvh * a.k_h + key0 * a.k_t;
    T const* vbase = static_cast<T const*>(a.v) + b * a.v_b + kvh * a.v_h + key0 * a.v_t;
    uint32_t const stage0 = smem_u32(smem);
    uint32_t const bar0 = smem_u32(bars);

    // Warp 0 issues the bulk copies of tile t (K tiles 0..ntile-1, then V tiles).
    auto issue = [&](int t) {
        bool const is_v = t >= ntile;
        int const lt = is_v ? t - ntile : t;
        int const rows = min(C::TILE, nkeys - lt * C::TILE);
        int64_t const stride = is_v ? a.v_t : a.k_t;
        T const* src = (is_v ? vbase : kbase) + static_cast<int64_t>(lt) * C::TILE * stride;
        int const s = t % kStages;
        uint32_t const bar = bar0 + s * 8;
        uint32_t const dst = stage0 + s * kStageBytes;
        if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(rows * C::ROWB));
        __syncwarp();
        if (stride == D) {
            if (lane == 0) bulk_copy_g2s(dst, src, static_cast<uint32_t>(rows * C::ROWB), bar);
        } else {
            for (int r = lane; r < rows; r += 32) bulk_copy_g2s(dst + r * C::ROWB, src + r * stride, C::ROWB, bar);
        }
    };

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(bar0 + s * 8, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == 0)
        for (int t = 0; t < min(kStages, total); ++t) issue(t);

    // This lane's slices of q for the score phase.
    int const sub = lane % C::LPK, grp = lane / C::LPK;
    V qr[C::VPL];
    {
        T const* qrow = static_cast<T const*>(a.q) + b * a.q_b + tq * a.q_t + hq * a.q_h;
#pragma unroll
        for (int m = 0; m < C::VPL; ++m) qr[m] = *reinterpret_cast<V const*>(qrow + (sub + C::LPK * m) * C::NV);
    }

    T mx = Lowest<T>::value;  // running max of this thread's scores
    T mrow = Lowest<T>::value, lrow = T{};
    V acc[C::VPLN];
#pragma unroll
    for (int m = 0; m < C::VPLN; ++m) acc[m] = V{};
    int const pv_key = C::VPR >= 32 ? 0 : lane / C::VPR;
    int const pv_vec = C::VPR >= 32 ? lane : lane % C::VPR;

    for (int t = 0; t < total; ++t) {
        int const s = t % kStages;
        bool const ok = mbar_wait_bounded(bar0 + s * 8, (t / kStages) & 1);
        // All threads agree on abort; the barrier also retires reads of tile t-1.
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                atomicOr(&g_decode_error, ANN_DEVERR_WAIT_TIMEOUT);
                // Drain the copies still in flight (bounded) before leaving.
                for (int u = t + 1; u < min(total, t - 1 + kStages); ++u)
                    mbar_wait_bounded(bar0 + (u % kStages) * 8, (u / kStages) & 1);
            }
            return;
        }
        if (t >= 1 && warp == 0 && t - 1 + kStages < total) issue(t - 1 + kStages);

        V const* tile = reinterpret_cast<V const*>(smem + s * kStageBytes);
        if (t < ntile) {
            int const kb = t * C::TILE;
            int const rows = min(C::TILE, nkeys - kb);
            for (int base = warp * C::KPW; base < rows; base += kWarps * C::KPW) {
                int const kk = base + grp;
                T part{};
                if (kk < rows) {
#pragma unroll
                    for (int m = 0; m < C::VPL; ++m) part = dot16<T>(qr[m], tile[kk * C::VPR + sub + C::LPK * m], part);
                }
#pragma unroll
                for (int o = C::LPK / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
                if (kk < rows && sub == 0) {
                    T const sv = part * scale;  // attentionScores, then ops::scale
                    sc[kb + kk] = sv;
                    mx = fmax(mx, sv);
                }
            }
        } else {
            if (t == ntile) {
                // softmax over this split's keys (all scores are in `sc`)
                mrow = block_max<kWarps>(mx, red_s);
                T ls{};
                for (int i = tid; i < nkeys; i += kThreads) {
                    T const p = exp_t(sc[i] - mrow);
                    sc[i] = p;
                    ls += p;
                }
                lrow = block_sum<kWarps>(ls, red_s);
            }
            int const kb = (t - ntile) * C::TILE;
            int const rows = min(C::TILE, nkeys - kb);
            for (int base = warp * C::KPS; base < rows; base += kWarps * C::KPS) {
                int const kk = base + pv_key;
                if (kk < rows) {
                    T const p = sc[kb + kk];
#pragma unroll
                    for (int m = 0; m < C::VPLN; ++m) axpy16<T>(acc[m], p, tile[kk * C::VPR + pv_vec + 32 * m]);
                }
            }
        }
    }

    // Reduce the per-warp partial sums: lanes holding the same vector first,
    // then the warps through shared memory (aliasing the drained stages).
    if constexpr (C::KPS > 1) {
#pragma unroll
        for (int m = 0; m < C::VPLN; ++m) {
#pragma unroll
            for (int o = C::VPR; o < 32; o <<= 1) {
                if constexpr (C::NV == 4) {
                    acc[m].x += __shfl_xor_sync(0xffffffffu, acc[m].x, o);
                    acc[m].y += __shfl_xor_sync(0xffffffffu, acc[m].y, o);
                    acc[m].z += __shfl_xor_sync(0xffffffffu, acc[m].z, o);
                    acc[m].w += __shfl_xor_sync(0xffffffffu, acc[m].w, o);
                } else {
                    acc[m].x += __shfl_xor_sync(0xffffffffu, acc[m].x, o);
                    acc[m].y += __shfl_xor_sync(0xffffffffu, acc[m].y, o);
                }
            }
        }
    }
    __syncthreads();
    T* red = reinterpret_cast<T*>(smem);
    if (lane < (C::VPR >= 32 ? 32 : C::VPR)) {
#pragma unroll
        for (int m = 0; m < C::VPLN; ++m)
            *reinterpret_cast<V*>(red + warp * D + (pv_vec + 32 * m) * C::NV) = acc[m];
    }
    __syncthreads();

    T* out = static_cast<T*>(a.out) + b * a.o_b + tq * a.o_t + hq * a.o_h;
    if (a.splits == 1) {
        for (int d = tid; d < D; d += kThreads) {
            T s{};
#pragma unroll
            for (int w = 0; w < kWarps; ++w) s += red[w * D + d];
            out[d * a.o_d] = lrow > T{} ? s / lrow : T{};
        }
        return;
    }

    T* pacc = static_cast<T*>(a.part_acc) + (row * a.splits) * D;
    T* pml = static_cast<T*>(a.part_ml) + (row * a.splits) * 2;
    for (int d = tid; d < D; d += kThreads) {
        T s{};
#pragma unroll
        for (int w = 0; w < kWarps; ++w) s += red[w * D + d];
        pacc[split * D + d] = s;
    }
    if (tid == 0) {
        pml[2 * split] = mrow;
        pml[2 * split + 1] = lrow;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(a.count + row, 1u) == static_cast<unsigned>(a.splits - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    T M = Lowest<T>::value;
    for (int s2 = 0; s2 < a.splits; ++s2) M = fmax(M, __ldcg(pml + 2 * s2));
    T L{};
    for (int s2 = 0; s2 < a.splits; ++s2) L += exp_t(__ldcg(pml + 2 * s2) - M) * __ldcg(pml + 2 * s2 + 1);
    for (int d = tid; d < D; d += kThreads) {
        T o{};
        for (int s2 = 0; s2 < a.splits; ++s2) o += exp_t(__ldcg(pml + 2 * s2) - M) * __ldcg(pacc + s2 * D + d);
        out[d * a.o_d] = L > T{} ? o / L : T{};
    }
    if (tid == 0) a.count[row] = 0u;  // leave the workspace ready for the next call
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct WsLayout {
    size_t acc, ml, count, total;
};

WsLayout ws_layout(int64_t rows, int64_t D, size_t eb) {
    WsLayout w{};
    w.acc = 0;
    w.ml = align256(static_cast<size_t>(rows) * kMaxSplits * D * eb);
    w.count = w.ml + align256(static_cast<size_t>(rows) * kMaxSplits * 2 * eb);
    w.total = w.count + static_cast<size_t>(rows) * sizeof(unsigned int);
    return w;
}

// Splits per row: enough CTAs to fill every resident slot, chosen to keep the
// last wave full; keys per split a multiple of the tile, at most kMaxChunk.
int choose_splits(int64_t rows, int64_t Tk, int tile, int slots, int64_t& chunk) {
    if (Tk <= 0) {
        chunk = 1;
        return 1;
    }
    int64_t const max_s = std::min<int64_t>(kMaxSplits, ceil_div(Tk, tile));
    int64_t const min_s = ceil_div(Tk, kMaxChunk);
    if (const char* env = std::getenv("ANN_DECODE_SPLITS")) {
        int64_t s = std::atoll(env);
        if (s >= min_s && s <= max_s) {
            chunk = ceil_div(ceil_div(Tk, s), tile) * tile;
            return static_cast<int>(ceil_div(Tk, chunk));
        }
    }
    double best = -1.0;
    int best_s = static_cast<int>(min_s);
    int64_t best_chunk = ceil_div(ceil_div(Tk, min_s), tile) * tile;
    for (int64_t s = min_s; s <= max_s; ++s) {
        int64_t const c = ceil_div(ceil_div(Tk, s), tile) * tile;
        int64_t const real_s = ceil_div(Tk, c);
        if (real_s != s) continue;
        int64_t const ctas = rows * real_s;
        int64_t const waves = ceil_div(ctas, slots);
        double const eff = static_cast<double>(ctas) / static_cast<double>(waves * slots);
        if (eff > best + 0.02) {
            best = eff;
            best_s = static_cast<int>(real_s);
            best_chunk = c;
        }
    }
    chunk = best_chunk;
    return best_s;
}

template <typename T, int D>
int launch(ann_stream stream, DecodeArgs& a, T scale, void* ws, size_t ws_bytes) {
    using C = Cfg<T, D>;
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    static int occ = 0;
    std::call_once(once, [] {
        attr_err = cudaFuncSetAttribute(decode_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(C::SMEM));
        if (attr_err == cudaSuccess)
            attr_err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_kernel<T, D>, kThreads, C::SMEM);
    });
    if (attr_err != cudaSuccess) return fail(ANN_ECUDA, "attention decode setup: %s", cudaGetErrorString(attr_err));
    int const slots = std::max(1, occ) * sm_count();
    int64_t chunk = 0;
    a.splits = choose_splits(a.rows, a.Tk, C::TILE, slots, chunk);
    a.chunk = chunk;
    if (a.splits > kMaxSplits)
        return fail(ANN_ENOTSUP, "attention decode: more than %d keys per row not supported.", kMaxSplits * kMaxChunk);
    if (a.splits > 1) {
        WsLayout const w = ws_layout(a.rows, D, sizeof(T));
        if (ws == nullptr || ws_bytes < w.total || !aligned(ws, 256))
            return fail(ANN_EINVAL, "attention decode: workspace of %zu bytes (256-byte aligned) required.", w.total);
        char* base = static_cast<char*>(ws);
        a.part_acc = base + w.acc;
        a.part_ml = base + w.ml;
        a.count = reinterpret_cast<unsigned int*>(base + w.count);
    }
    int64_t const grid = a.rows * a.splits;
    if (grid > INT32_MAX) return fail(ANN_ENOTSUP, "attention decode: grid too large.");
    decode_kernel<T, D><<<static_cast<unsigned>(grid), kThreads, C::SMEM, as_stream(stream)>>>(a, scale);
    return check_launch("attention decode");
}

template <typename T>
int decode(ann_stream stream, const ann_view* q_v, const ann_view* k_v, const ann_view* v_v, const ann_view* o_v,
           T scale, uint32_t g, int layout, void* ws, size_t ws_bytes) {
    if (g == 0u) return fail(ANN_EINVAL, "attention decode requires queriesPerKvGroup > 0.");
    if (layout != ANN_LAYOUT_BTHD && layout != ANN_LAYOUT_BHTD)
        return fail(ANN_EINVAL, "attention decode: invalid kv layout.");
    Dims q, k, v, o;
    ANN_TRY(to_dims(q_v, sizeof(T), "attention decode Q", q));
    ANN_TRY(to_dims(k_v, sizeof(T), "attention decode K", k));
    ANN_TRY(to_dims(v_v, sizeof(T), "attention decode V", v));
    ANN_TRY(to_dims(o_v, sizeof(T), "attention decode out", o));
    if (q.rank != 4 || k.rank != 4 || v.rank != 4 || o.rank != 4)
        return fail(ANN_EINVAL, "attention decode expects rank-4 tensors.");
    if (!same_extents(q, o)) return fail(ANN_EINVAL, "attention decode: out must have the extents of Q.");
    if (!same_extents(k, v)) return fail(ANN_EINVAL, "attention decode: K and V extents differ.");
    int const tok = layout == ANN_LAYOUT_BTHD ? 1 : 2, head = layout == ANN_LAYOUT_BTHD ? 2 : 1;
    int64_t const B = q.ext[0], Tq = q.ext[1], Hq = q.ext[2], D = q.ext[3];
    if (k.ext[0] != B || k.ext[3] != D || k.ext[head] <= (Hq - 1) / static_cast<int64_t>(g))
        return fail(ANN_EINVAL, "attention decode: Q %s does not match K/V %s.", extents_str(q).c_str(),
                    extents_str(k).c_str());
    if (q.numel() == 0) return ANN_OK;
    bool const d_ok = sizeof(T) == 4 ? (D == 64 || D == 128 || D == 256) : (D == 64 || D == 128);
    if (!d_ok) return fail(ANN_ENOTSUP, "attention decode: head dim %lld not supported.", static_cast<long long>(D));
    size_t const eb = sizeof(T);
    bool const unit = q.str[3] == 1 && k.str[3] == 1 && v.str[3] == 1;
    bool const kv_aligned = aligned(k.data, 16) && aligned(v.data, 16) && (k.str[0] * eb) % 16 == 0 &&
                            (k.str[1] * eb) % 16 == 0 && (k.str[2] * eb) % 16 == 0 && (v.str[0] * eb) % 16 == 0 &&
                            (v.str[1] * eb) % 16 == 0 && (v.str[2] * eb) % 16 == 0;
    bool const q_aligned =
        aligned(q.data, 16) && (q.str[0] * eb) % 16 == 0 && (q.str[1] * eb) % 16 == 0 && (q.str[2] * eb) % 16 == 0;
    if (!unit || !kv_aligned || !q_aligned)
        return fail(ANN_ENOTSUP, "attention decode needs unit-stride head vectors and 16-byte aligned rows.");

    DecodeArgs a{};
    a.q = q.data;
    a.k = k.data;
    a.v = v.data;
    a.out = o.data;
    a.q_b = q.str[0];
    a.q_t = q.str[1];
    a.q_h = q.str[2];
    a.o_b = o.str[0];
    a.o_t = o.str[1];
    a.o_h = o.str[2];
    a.o_d = o.str[3];
    a.k_b = k.str[0];
    a.k_h = k.str[head];
    a.k_t = k.str[tok];
    a.v_b = v.str[0];
    a.v_h = v.str[head];
    a.v_t = v.str[tok];
    a.Tq = Tq;
    a.Hq = Hq;
    a.Tk = k.ext[tok];
    a.rows = B * Tq * Hq;
    a.g = g;
    if (sizeof(T) == 4) {
        if (D == 64) return launch<T, 64>(stream, a, scale, ws, ws_bytes);
        if (D == 128) return launch<T, 128>(stream, a, scale, ws, ws_bytes);
        return launch<T, (sizeof(T) == 4 ? 256 : 128)>(stream, a, scale, ws, ws_bytes);
    }
    if (D == 64) return launch<T, 64>(stream, a, scale, ws, ws_bytes);
    return launch<T, 128>(stream, a, scale, ws, ws_bytes);
}

}  // namespace

int take_decode_error(cudaStream_t s, uint32_t* bits) {
    unsigned int value = 0, zero = 0;
    if (cudaMemcpyFromSymbolAsync(&value, g_decode_error, sizeof value, 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_decode_error, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ANN_ECUDA, "device error word: %s", cudaGetErrorString(cudaGetLastError()));
    *bits |= value;
    return ANN_OK;
}

}  // namespace ann

extern "C" {

size_t ann_attention_decode_workspace_size(int64_t batch, int64_t query_tokens, int64_t query_heads,
                                           int64_t head_dim, int64_t kv_tokens, int32_t elem_bytes) {
    (void)kv_tokens;
    if (batch < 0 || query_tokens < 0 || query_heads < 0 || head_dim < 0 || (elem_bytes != 4 && elem_bytes != 8))
        return 0;
    return ann::ws_layout(batch * query_tokens * query_heads, head_dim, static_cast<size_t>(elem_bytes)).total;
}

int ann_attention_decode_f32(ann_stream s, const ann_view* q, const ann_view* k, const ann_view* v,
                             const ann_view* out, float scale, uint32_t g, int32_t layout, void* ws,
                             size_t ws_bytes) {
    ANN_API_BEGIN
    return ann::decode<float>(s, q, k, v, out, scale, g, layout, ws, ws_bytes);
    ANN_API_END
}

int ann_attention_decode_f64(ann_stream s, const ann_view* q, const ann_view* k, const ann_view* v,
                             const ann_view* out, double scale, uint32_t g, int32_t layout, void* ws,
                             size_t ws_bytes) {
    ANN_API_BEGIN
    return ann::decode<double>(s, q, k, v, out, scale, g, layout, ws, ws_bytes);
    ANN_API_END
}

}  // extern "C"
