// decode.cu -- fused decode attention over a KV cache (split-K, cluster merge).
//
// Computes in ONE launch what the reference's decode pipeline computes in four
// (test/unit/nn/attention.cpp:675-734):
//   attentionScores (onAcc/internal/nn/attention.hpp:21-39)
//   -> ops::scale (onHost/ops/elementwise.hpp:64-73)
//   -> softmax over all keys (onAcc/internal/nn/softmax.hpp:32-74, non-causal)
//   -> attentionApply (onAcc/internal/nn/attention.hpp:49-67)
// without writing the [B,Hq,Tq,Tk] score and probability tensors to memory.
//
// The work is memory-bound (each K/V byte feeds one FMA), so the design is
// about streaming the cache at HBM rate with no extra traffic:
//  * one thread-block CLUSTER of S CTAs per query row (batch, query token,
//    query head); CTA s of the cluster owns a contiguous key range of the
//    row's KV head (GQA: hq / g);
//  * K and V rows are streamed through a 4-stage ring of 16 KB shared-memory
//    tiles by 1-D bulk copies (TMA, cp.async.bulk, never multicast)
//    completing on mbarriers;
//  * keys are taken in sub-chunks of up to 2048: the sub-chunk's K tiles give
//    its scores (8 lanes per key, 16-byte slices, 3-shuffle reduction, kept
//    in shared memory), then its exact max / exp / sum, then its V tiles
//    accumulate sum(p * v). Sub-chunks merge into a running (max, sum, acc)
//    with the online-softmax rescale, so any cache length is handled;
//  * the S partial results of a row meet in distributed shared memory: each
//    CTA merges one slice of the head dimension from all S peers with the
//    log-sum-exp rule  out = sum_s e^(m_s-M) acc_s / sum_s e^(m_s-M) l_s.
//    No global scratch memory, no atomics, no second launch.
// Summation order differs from the reference's sequential loops (tree
// reductions, split merge); results agree within the fp32/fp64 tolerances.
#include <cooperative_groups.h>

#include <array>
#include <cstdlib>
#include <map>
#include <mutex>

#include "common.cuh"
#include "multimem.cuh"
#include "reduce.cuh"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace ann {
namespace {

__device__ unsigned int g_decode_error;

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 4;
constexpr int kStageBytes = 16384;
constexpr int kSub = 2048;       // keys per sub-chunk (scores kept in shared memory)
constexpr int kMaxCluster = 16;  // splits per row (non-portable cluster size)

struct DecodeArgs {
    const void* q;
    const void* k;
    const void* v;
    void* out;
    void* mirror;                // multicast address of out[0] (stores reach every rank's copy), or null
    int64_t q_b, q_t, q_h;       // element strides of Q (unit stride along d)
    int64_t o_b, o_t, o_h, o_d;  // element strides of out
    int64_t k_b, k_h, k_t;       // element strides of K by batch, kv head, token
    int64_t v_b, v_h, v_t;
    int64_t Tq, Hq, Tk, chunk, rows;
    uint32_t g;
    int splits;
};

template <typename T, int D>
struct Cfg {
    using V = typename Vec16<T>::type;
    static constexpr int NV = Vec16<T>::n;
    static constexpr int ROWB = D * static_cast<int>(sizeof(T));  // bytes per key row
    static constexpr int VPR = ROWB / 16;                         // 16-byte vectors per row
    static constexpr int TILE = kStageBytes / ROWB;               // keys per stage
    static constexpr int TPS = kSub / TILE;                       // tiles per full sub-chunk
    static constexpr int LPK = 8;                                 // score phase: lanes per key
    static constexpr int KPW = 32 / LPK;                          // keys per warp step
    static constexpr int VPL = VPR / LPK;                         // vectors per lane per key
    static constexpr int KPS = VPR >= 32 ? 1 : 32 / VPR;          // PV phase: keys per warp step
    static constexpr int VPLN = VPR >= 32 ? VPR / 32 : 1;         // PV phase: vectors per lane
    static constexpr size_t OFF_SC = kStages * kStageBytes;
    static constexpr size_t OFF_BAR = OFF_SC + kSub * sizeof(T);
    static constexpr size_t OFF_XCH = OFF_BAR + kStages * sizeof(uint64_t);
    static constexpr size_t SMEM = OFF_XCH + (D + 2) * sizeof(T);
    static_assert(ROWB % 128 == 0, "row must be a multiple of 128 bytes");
    static_assert(kSub % TILE == 0, "sub-chunk must be whole tiles");
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

template <typename T>
__device__ __forceinline__ void scale16(typename Vec16<T>::type& acc, T f);
template <>
__device__ __forceinline__ void scale16<float>(float4& acc, float f) {
    acc.x *= f;
    acc.y *= f;
    acc.z *= f;
    acc.w *= f;
}
template <>
__device__ __forceinline__ void scale16<double>(double2& acc, double f) {
    acc.x *= f;
    acc.y *= f;
}

template <typename T>
__device__ __forceinline__ void shfl_add16(typename Vec16<T>::type& acc, int o) {
    if constexpr (Vec16<T>::n == 4) {
        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
        acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
        acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
    } else {
        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
    }
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) decode_kernel(DecodeArgs a, T scale) {
    using C = Cfg<T, D>;
    using V = typename C::V;
    extern __shared__ __align__(128) unsigned char smem[];
    T* sc = reinterpret_cast<T*>(smem + C::OFF_SC);
    T* xch = reinterpret_cast<T*>(smem + C::OFF_XCH);  // this CTA's [acc(D), m, l] for the cluster merge
    __shared__ T red_s[kWarps];

    int const tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int const split = static_cast<int>(blockIdx.x % a.splits);  // == rank in the cluster
    int64_t const row = blockIdx.x / a.splits;
    int64_t const hq = row % a.Hq;
    int64_t const tq = (row / a.Hq) % a.Tq;
    int64_t const b = row / (a.Hq * a.Tq);
    int64_t const kvh = hq / a.g;
    int64_t const key0 = static_cast<int64_t>(split) * a.chunk;
    int64_t const left = a.Tk - key0;
    int const n = static_cast<int>(left <= 0 ? 0 : (left < a.chunk ? left : a.chunk));
    int const total = 2 * ((n + C::TILE - 1) / C::TILE);

    T const* kbase = static_cast<T const*>(a.k) + b * a.k_b + kvh * a.k_h + key0 * a.k_t;
    T const* vbase = static_cast<T const*>(a.v) + b * a.v_b + kvh * a.v_h + key0 * a.v_t;
    uint32_t const stage0 = smem_u32(smem);
    uint32_t const bar0 = smem_u32(smem + C::OFF_BAR);

    // Tile t of the stream K(sub 0), V(sub 0), K(sub 1), V(sub 1), ...
    struct TileInfo {
        int sub, nc, lt, rows;
        bool is_v;
    };
    auto tile_info = [&](int t) {
        TileInfo ti;
        ti.sub = t / (2 * C::TPS);
        int const within = t - ti.sub * 2 * C::TPS;
        ti.nc = min(kSub, n - ti.sub * kSub);
        int const ntc = (ti.nc + C::TILE - 1) / C::TILE;
        ti.is_v = within >= ntc;
        ti.lt = ti.is_v ? within - ntc : within;
        ti.rows = min(C::TILE, ti.nc - ti.lt * C::TILE);
        return ti;
    };

    // Warp 0 issues the bulk copies of tile t into stage t % kStages.
    auto issue = [&](int t) {
        TileInfo const ti = tile_info(t);
        int64_t const stride = ti.is_v ? a.v_t : a.k_t;
        int64_t const key = static_cast<int64_t>(ti.sub) * kSub + static_cast<int64_t>(ti.lt) * C::TILE;
        T const* src = (ti.is_v ? vbase : kbase) + key * stride;
        int const s = t % kStages;
        uint32_t const bar = bar0 + s * 8;
        uint32_t const dst = stage0 + s * kStageBytes;
        if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(ti.rows * C::ROWB));
        __syncwarp();
        if (stride == D) {
            if (lane == 0) bulk_copy_g2s(dst, src, static_cast<uint32_t>(ti.rows * C::ROWB), bar);
        } else {
            for (int r = lane; r < ti.rows; r += 32)
                bulk_copy_g2s(dst + r * C::ROWB, src + r * stride, C::ROWB, bar);
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

    T mx = Lowest<T>::value;  // max of this thread's scores in the current sub-chunk
    T m_run = Lowest<T>::value, l_run = T{};
    V acc[C::VPLN];
#pragma unroll
    for (int m = 0; m < C::VPLN; ++m) acc[m] = V{};
    int const pv_key = C::VPR >= 32 ? 0 : lane / C::VPR;
    int const pv_vec = C::VPR >= 32 ? lane : lane % C::VPR;

    for (int t = 0; t < total; ++t) {
        int const s = t % kStages;
        bool const ok = mbar_wait_bounded(bar0 + s * 8, (t / kStages) & 1);
        // All threads agree on abort; the barrier also retires the reads of tile t-1.
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                atomicOr(&g_decode_error, ANN_DEVERR_WAIT_TIMEOUT);
                // drain every copy still in flight, tile t's own included, before
                // the stages are reused as reduction scratch (each wait bounded)
                for (int u = t; u < min(total, t - 1 + kStages); ++u)
                    mbar_wait_bounded(bar0 + (u % kStages) * 8, (u / kStages) & 1);
            }
            break;  // still joins the cluster barriers below
        }
        if (t >= 1 && warp == 0 && t - 1 + kStages < total) issue(t - 1 + kStages);

        TileInfo const ti = tile_info(t);
        V const* tile = reinterpret_cast<V const*>(smem + s * kStageBytes);
        int const kb = ti.lt * C::TILE;
        if (!ti.is_v) {
            for (int base = warp * C::KPW; base < ti.rows; base += kWarps * C::KPW) {
                int const kk = base + grp;
                T part{};
                if (kk < ti.rows) {
#pragma unroll
                    for (int m = 0; m < C::VPL; ++m) part = dot16<T>(qr[m], tile[kk * C::VPR + sub + C::LPK * m], part);
                }
#pragma unroll
                for (int o = C::LPK / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
                if (kk < ti.rows && sub == 0) {
                    T const sv = part * scale;  // attentionScores, then ops::scale
                    sc[kb + kk] = sv;
                    mx = fmax(mx, sv);
                }
            }
        } else {
            if (ti.lt == 0) {
                // softmax statistics of this sub-chunk, merged into the running ones
                T const m_c = block_max<kWarps>(mx, red_s);
                T const m_new = fmax(m_run, m_c);
                T const alpha = exp_t(m_run - m_new);
#pragma unroll
                for (int m = 0; m < C::VPLN; ++m) scale16<T>(acc[m], alpha);
                T ls{};
                for (int i = tid; i < ti.nc; i += kThreads) {
                    T const p = exp_t(sc[i] - m_new);
                    sc[i] = p;
                    ls += p;
                }
                l_run = l_run * alpha + block_sum<kWarps>(ls, red_s);
                m_run = m_new;
                mx = Lowest<T>::value;
            }
            for (int base = warp * C::KPS; base < ti.rows; base += kWarps * C::KPS) {
                int const kk = base + pv_key;
                if (kk < ti.rows) {
                    T const p = sc[kb + kk];
#pragma unroll
                    for (int m = 0; m < C::VPLN; ++m) axpy16<T>(acc[m], p, tile[kk * C::VPR + pv_vec + 32 * m]);
                }
            }
        }
    }

    // Per-CTA result: lanes holding the same vector first, then the warps
    // through shared memory (aliasing the drained stages).
    if constexpr (C::KPS > 1) {
#pragma unroll
        for (int m = 0; m < C::VPLN; ++m)
#pragma unroll
            for (int o = C::VPR; o < 32; o <<= 1) shfl_add16<T>(acc[m], o);
    }
    __syncthreads();
    T* red = reinterpret_cast<T*>(smem);
    if (lane < (C::VPR >= 32 ? 32 : C::VPR)) {
#pragma unroll
        for (int m = 0; m < C::VPLN; ++m)
            *reinterpret_cast<V*>(red + warp * D + (pv_vec + 32 * m) * C::NV) = acc[m];
    }
    __syncthreads();
    int64_t const out_off = b * a.o_b + tq * a.o_t + hq * a.o_h;
    T* out = static_cast<T*>(a.out) + out_off;
    T* mout = a.mirror ? static_cast<T*>(a.mirror) + out_off : nullptr;
    if (a.splits == 1) {
        for (int d = tid; d < D; d += kThreads) {
            T s{};
#pragma unroll
            for (int w = 0; w < kWarps; ++w) s += red[w * D + d];
            T const val = l_run > T{} ? s / l_run : T{};
            if (mout) mc::store(mout + d * a.o_d, val);
            else out[d * a.o_d] = val;
        }
        return;
    }
    for (int d = tid; d < D; d += kThreads) {
        T s{};
#pragma unroll
        for (int w = 0; w < kWarps; ++w) s += red[w * D + d];
        xch[d] = s;
    }
    if (tid == 0) {
        xch[D] = m_run;
        xch[D + 1] = l_run;
    }

    // Merge the cluster's partial results through distributed shared memory:
    // CTA `split` produces the output dims [lo, hi).
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    int const per = (D + a.splits - 1) / a.splits;
    int const lo = split * per, hi = min(D, lo + per);
    if (tid < hi - lo) {
        T M = Lowest<T>::value;
        for (int r = 0; r < a.splits; ++r) M = fmax(M, cluster.map_shared_rank(xch, r)[D]);
        T L{}, o{};
        for (int r = 0; r < a.splits; ++r) {
            T const* px = cluster.map_shared_rank(xch, r);
            T const w = exp_t(px[D] - M);
            L += w * px[D + 1];
            o += w * px[lo + tid];
        }
        T const val = L > T{} ? o / L : T{};
        if (mout) mc::store(mout + (lo + tid) * a.o_d, val);
        else out[(lo + tid) * a.o_d] = val;
    }
    cluster.sync();  // peers' shared memory must outlive the reads above
}

// Splits per row = cluster size. The kernel is HBM-bound, so what matters is
// (a) enough CTAs streaming at once (each keeps 64 KB in flight) and (b) no
// short last wave of long CTAs, during which HBM idles. Rule: the smallest
// split count s with
//   * rows*s >= ~1.7 CTAs per SM,
//   * at most 16384 keys per CTA, and
//   * a single wave (rows*s <= resident slots) or a last wave that is full or
//     holds >= ~1.7 CTAs per SM;
// else the smallest s meeting the first two. Measured on B200 (148 SMs, 3
// resident CTAs each) this picks the fastest or within 3 % of the fastest
// split at every row count tried: 32..256 rows of 2048 keys, 128..1024 rows
// of 32768 keys (e.g. 256 rows of 32768 keys: 1 split 6.6 TB/s, 2 splits
// 5.5 TB/s with a 68-CTA last wave, 3 splits 7.1 TB/s).
template <typename T, int D>
int choose_splits(int64_t rows, int64_t Tk, int64_t& chunk, const int* slots_for) {
    using C = Cfg<T, D>;
    if (Tk <= 0) {
        chunk = 1;
        return 1;
    }
    auto realize = [&](int64_t s) {
        chunk = ceil_div(ceil_div(Tk, s), C::TILE) * C::TILE;
        return static_cast<int>(ceil_div(Tk, chunk));
    };
    if (const char* env = std::getenv("ANN_DECODE_SPLITS")) {
        int s = std::atoi(env);
        if (s >= 1 && s <= kMaxCluster && slots_for[s] > 0) return realize(s);
    }
    int64_t const max_s = std::max<int64_t>(1, std::min<int64_t>(kMaxCluster, Tk / (4 * C::TILE)));
    int64_t const target = (17 * static_cast<int64_t>(sm_count()) + 9) / 10;
    int64_t fallback = 0;
    for (int64_t s = 1; s <= max_s; ++s) {
        if (slots_for[s] <= 0) continue;
        int64_t const ctas = rows * s;
        bool const enough = ctas >= target || s == max_s;
        bool const short_ctas = ceil_div(Tk, s) <= 16384 || s == max_s;
        if (!enough || !short_ctas) continue;
        if (fallback == 0) fallback = s;
        int64_t const tail = ctas % slots_for[s];
        if (ctas <= slots_for[s] || tail == 0 || tail >= target) return realize(s);
    }
    return realize(fallback > 0 ? fallback : 1);
}

template <typename T, int D>
int launch(ann_stream stream, DecodeArgs& a, T scale) {
    using C = Cfg<T, D>;
    static std::mutex mu;
    static std::map<int, std::array<int, kMaxCluster + 1>> slots_by_dev;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(ANN_ECUDA, "attention decode: no CUDA device.");
    std::array<int, kMaxCluster + 1> slots{};
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = slots_by_dev.find(dev);
        if (it == slots_by_dev.end()) {
            cudaError_t e = cudaFuncSetAttribute(decode_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(C::SMEM));
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(decode_kernel<T, D>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return fail(ANN_ECUDA, "attention decode setup: %s", cudaGetErrorString(e));
            for (int s = 1; s <= kMaxCluster; ++s) {
                cudaLaunchConfig_t cfg{};
                cudaLaunchAttribute attr{};
                attr.id = cudaLaunchAttributeClusterDimension;
                attr.val.clusterDim.x = s;
                attr.val.clusterDim.y = 1;
                attr.val.clusterDim.z = 1;
                cfg.gridDim = dim3(s * 1024);
                cfg.blockDim = dim3(kThreads);
                cfg.dynamicSmemBytes = C::SMEM;
                cfg.attrs = &attr;
                cfg.numAttrs = 1;
                int clusters = 0;
                if (cudaOccupancyMaxActiveClusters(&clusters, decode_kernel<T, D>, &cfg) != cudaSuccess) {
                    cudaGetLastError();
                    clusters = 0;
                }
                slots[s] = clusters * s;
            }
            if (slots[1] <= 0) return fail(ANN_ECUDA, "attention decode: kernel does not fit on this device.");
            slots_by_dev[dev] = slots;
        } else {
            slots = it->second;
        }
    }
    int64_t chunk = 0;
    a.splits = choose_splits<T, D>(a.rows, a.Tk, chunk, slots.data());
    a.chunk = chunk;
    int64_t const grid = a.rows * a.splits;
    if (grid > INT32_MAX) return fail(ANN_ENOTSUP, "attention decode: grid too large.");
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = static_cast<unsigned>(a.splits);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = as_stream(stream);
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    cudaError_t const e = cudaLaunchKernelEx(&cfg, decode_kernel<T, D>, a, scale);
    if (e != cudaSuccess) return fail(ANN_ECUDA, "attention decode: %s", cudaGetErrorString(e));
    return check_launch("attention decode");
}

template <typename T>
int decode(ann_stream stream, const ann_view* q_v, const ann_view* k_v, const ann_view* v_v, const ann_view* o_v,
           T scale, uint32_t g, int layout, void* mirror = nullptr) {
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
    a.mirror = mirror;
    if (mirror != nullptr && !aligned(mirror, sizeof(T)))
        return fail(ANN_EINVAL, "attention decode: the output mirror is misaligned.");
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
    if constexpr (sizeof(T) == 4) {
        if (D == 64) return launch<T, 64>(stream, a, scale);
        if (D == 128) return launch<T, 128>(stream, a, scale);
        return launch<T, 256>(stream, a, scale);
    } else {
        if (D == 64) return launch<T, 64>(stream, a, scale);
        return launch<T, 128>(stream, a, scale);
    }
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

int ann_attention_decode_f32(ann_stream s, const ann_view* q, const ann_view* k, const ann_view* v,
                             const ann_view* out, float scale, uint32_t g, int32_t layout) {
    ANN_API_BEGIN
    return ann::decode<float>(s, q, k, v, out, scale, g, layout);
    ANN_API_END
}

int ann_attention_decode_f64(ann_stream s, const ann_view* q, const ann_view* k, const ann_view* v,
                             const ann_view* out, double scale, uint32_t g, int32_t layout) {
    ANN_API_BEGIN
    return ann::decode<double>(s, q, k, v, out, scale, g, layout);
    ANN_API_END
}

int ann_attention_decode_mirror_f32(ann_stream s, const ann_view* q, const ann_view* k, const ann_view* v,
                                    const ann_view* out, void* out_mirror, float scale, uint32_t g,
                                    int32_t layout) {
    ANN_API_BEGIN
    if (out_mirror == nullptr) return ann::fail(ANN_EINVAL, "attention decode: the output mirror is NULL.");
    return ann::decode<float>(s, q, k, v, out, scale, g, layout, out_mirror);
    ANN_API_END
}

int ann_attention_decode_mirror_f64(ann_stream s, const ann_view* q, const ann_view* k, const ann_view* v,
                                    const ann_view* out, void* out_mirror, double scale, uint32_t g,
                                    int32_t layout) {
    ANN_API_BEGIN
    if (out_mirror == nullptr) return ann::fail(ANN_EINVAL, "attention decode: the output mirror is NULL.");
    return ann::decode<double>(s, q, k, v, out, scale, g, layout, out_mirror);
    ANN_API_END
}

}  // extern "C"
