// prefill.cu -- fused prefill attention, register-tiled on the FMA / DFMA pipes.
//
// Computes in ONE launch the reference's prefill pipeline
// (test/unit/nn/attention.cpp:591-651):
//   attentionScores (onAcc/internal/nn/attention.hpp:21-39)
//   -> ops::scale (onHost/ops/elementwise.hpp:64-73)
//   -> causalSoftmax, top-left mask key > query (onAcc/internal/nn/softmax.hpp:23-74)
//      or softmax (non-causal)
//   -> attentionApply (onAcc/internal/nn/attention.hpp:49-67)
// without materialising the [B,Hq,Tq,Tk] scores / probabilities.
//
// This is the SIMT path (FMA / DFMA), used when ANN_PREFILL_FMA=1 asks for it or
// the tensor-core kernels (prefill_tc.cu for fp32, prefill_f64.cu for fp64)
// cannot take the shape. One CTA owns 64 query
// rows of one (batch, query head); K/V tiles of 64 keys stream through two
// shared-memory stages filled by 1-D bulk copies (one per 16-byte aligned
// row, rows padded by 16 bytes so the column-wise reads are bank-conflict
// free). Each thread holds a 4x4 block of the score tile (query rows
// ty+16m, keys tx+16n), keeps the online softmax statistics of its 4 rows
// (reduced over the 16 lanes that share them), and accumulates 4 rows x D/16
// output columns of P.V. Causal tiles above the diagonal are skipped; CTAs
// with the most key tiles are dispatched first.
#include <mutex>

#include <cstdlib>

#include "common.cuh"
#include "reduce.cuh"
#include "tma.cuh"

namespace ann {

int prefill_tc_f32(ann_stream stream, const Dims& q, const Dims& k, const Dims& v, const Dims& o, float scale,
                   uint32_t g, int layout, int causal, bool& handled);
int prefill_tc_pair_f32(ann_stream stream, const Dims& q, const Dims& k, const Dims& v, const Dims& o, float scale,
                        uint32_t g, int layout, int causal, bool& handled, void* mirror);
int prefill_mma_f64(ann_stream stream, const Dims& q, const Dims& k, const Dims& v, const Dims& o, double scale,
                    uint32_t g, int layout, int causal, bool& handled, void* mirror);

namespace {

__device__ unsigned int g_prefill_error;

constexpr int kBM = 64, kThreads = 256;

__device__ __forceinline__ int64_t min64(int64_t x, int64_t y) { return x < y ? x : y; }

struct PrefillArgs {
    const void* q;
    const void* k;
    const void* v;
    void* out;
    int64_t q_b, q_t, q_h;       // element strides of Q (unit stride along d)
    int64_t o_b, o_t, o_h, o_d;  // element strides of out
    int64_t k_b, k_h, k_t;
    int64_t v_b, v_h, v_t;
    int64_t Tq, Tk, Hq;
    uint32_t g;
    int causal;
    int q_tiles;
    int64_t bhs;         // batch * query heads
    int64_t head_chunk;  // (batch, head) pairs per dispatch chunk
};

template <typename T, int D, int BN>
struct PCfg {
    using V = typename Vec16<T>::type;
    static constexpr int NV = Vec16<T>::n;
    static constexpr int PAD = NV;                 // 16 bytes of padding per row
    static constexpr int LD = D + PAD;             // row pitch in elements
    static constexpr int LDP = BN + PAD;           // probability tile pitch
    static constexpr int KN = BN / 16;             // keys per thread in a score tile
    static constexpr int W = D / (16 * NV);        // output vectors per thread per row
    static constexpr int ROWB = D * static_cast<int>(sizeof(T));
    static constexpr size_t TILE_ELEMS = static_cast<size_t>(BN) * LD;
    static constexpr size_t OFF_Q = 0;
    static constexpr size_t OFF_K = OFF_Q + kBM * LD * sizeof(T);
    static constexpr size_t OFF_V = OFF_K + 2 * TILE_ELEMS * sizeof(T);
    static constexpr size_t OFF_P = OFF_V + 2 * TILE_ELEMS * sizeof(T);
    static constexpr size_t OFF_BAR = OFF_P + kBM * LDP * sizeof(T);
    static constexpr size_t SMEM = OFF_BAR + 3 * sizeof(uint64_t);
    static_assert(D % (16 * NV) == 0, "head dim must be a multiple of 16 vectors");
    static_assert((LD * sizeof(T)) % 128 == 16, "row pitch = 16 mod 128 bytes keeps column reads conflict-free");
};

template <typename T>
__device__ __forceinline__ T dotv(typename Vec16<T>::type a, typename Vec16<T>::type b, T acc) {
    if constexpr (Vec16<T>::n == 4) {
        acc = fma(a.x, b.x, acc);
        acc = fma(a.y, b.y, acc);
        acc = fma(a.z, b.z, acc);
        return fma(a.w, b.w, acc);
    } else {
        acc = fma(a.x, b.x, acc);
        return fma(a.y, b.y, acc);
    }
}

template <typename T>
__device__ __forceinline__ void axpyv(typename Vec16<T>::type& acc, T p, typename Vec16<T>::type v) {
    if constexpr (Vec16<T>::n == 4) {
        acc.x = fma(p, v.x, acc.x);
        acc.y = fma(p, v.y, acc.y);
        acc.z = fma(p, v.z, acc.z);
        acc.w = fma(p, v.w, acc.w);
    } else {
        acc.x = fma(p, v.x, acc.x);
        acc.y = fma(p, v.y, acc.y);
    }
}

template <typename T>
__device__ __forceinline__ T half_max(T v) {  // over the 16 lanes sharing query rows
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
template <typename T>
__device__ __forceinline__ T half_sum(T v) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <typename T, int D, int BN>
__global__ void __launch_bounds__(kThreads) prefill_kernel(PrefillArgs a, T scale) {
    using C = PCfg<T, D, BN>;
    constexpr int kBN = BN;
    using V = typename C::V;
    extern __shared__ __align__(128) unsigned char smem[];
    T* Qs = reinterpret_cast<T*>(smem + C::OFF_Q);
    T* Ks = reinterpret_cast<T*>(smem + C::OFF_K);
    T* Vs = reinterpret_cast<T*>(smem + C::OFF_V);
    T* Ps = reinterpret_cast<T*>(smem + C::OFF_P);
    uint32_t const bar0 = smem_u32(smem + C::OFF_BAR);  // [0] Q, [1] stage 0, [2] stage 1

    int const tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int const tx = tid & 15, ty = tid >> 4;
    // 1-D grid in chunks of a.head_chunk (batch, head) pairs (head_chunk_for):
    // inside a chunk the query tiles go from the last (most keys) down, so the
    // heaviest CTAs start first, while the K/V of one chunk stay in L2
    int64_t const lin = blockIdx.x, per_chunk = a.head_chunk * a.q_tiles;
    int64_t const chunk = lin / per_chunk, in_chunk = lin % per_chunk;
    int64_t const chunk_bh = a.bhs - chunk * a.head_chunk < a.head_chunk ? a.bhs - chunk * a.head_chunk : a.head_chunk;
    int const qt = a.q_tiles - 1 - static_cast<int>(in_chunk / chunk_bh);
    int64_t const bh = chunk * a.head_chunk + in_chunk % chunk_bh;
    int64_t const hq = bh % a.Hq, b = bh / a.Hq, kvh = hq / a.g;
    int64_t const q0 = static_cast<int64_t>(qt) * kBM;
    int const q_rows = static_cast<int>(min64(kBM, a.Tq - q0));
    int64_t const k_end = a.causal ? min64(a.Tk, q0 + kBM) : a.Tk;  // keys <= last query of the tile
    int const n_kt = static_cast<int>((k_end + kBN - 1) / kBN);

    T const* qbase = static_cast<T const*>(a.q) + b * a.q_b + q0 * a.q_t + hq * a.q_h;
    T const* kbase = static_cast<T const*>(a.k) + b * a.k_b + kvh * a.k_h;
    T const* vbase = static_cast<T const*>(a.v) + b * a.v_b + kvh * a.v_h;

    auto issue_kv = [&](int kt) {  // warp 0: K and V rows of key tile kt into stage kt & 1
        int const s = kt & 1;
        int const rows = static_cast<int>(min64(kBN, a.Tk - static_cast<int64_t>(kt) * kBN));
        uint32_t const bar = bar0 + 8 * (1 + s);
        if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(2 * rows * C::ROWB));
        __syncwarp();
        uint32_t const kd = smem_u32(Ks + s * C::TILE_ELEMS), vd = smem_u32(Vs + s * C::TILE_ELEMS);
        for (int r = lane; r < rows; r += 32) {
            int64_t const key = static_cast<int64_t>(kt) * kBN + r;
            bulk_copy_g2s(kd + r * C::LD * sizeof(T), kbase + key * a.k_t, C::ROWB, bar);
            bulk_copy_g2s(vd + r * C::LD * sizeof(T), vbase + key * a.v_t, C::ROWB, bar);
        }
    };

    if (tid == 0) {
        for (int i = 0; i < 3; ++i) mbar_init(bar0 + 8 * i, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == 0) {
        if (lane == 0) mbar_arrive_expect_tx(bar0, static_cast<uint32_t>(q_rows * C::ROWB));
        __syncwarp();
        for (int r = lane; r < q_rows; r += 32)
            bulk_copy_g2s(smem_u32(Qs + r * C::LD), qbase + r * a.q_t, C::ROWB, bar0);
        for (int kt = 0; kt < min(2, n_kt); ++kt) issue_kv(kt);
    }
    // rows past the end of Q: zeros (never written out)
    for (int i = tid; i < (kBM - q_rows) * C::LD; i += kThreads) Qs[q_rows * C::LD + i] = T{};

    T m_run[4], l_run[4];
    V o[4][C::W];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        m_run[m] = Lowest<T>::value;
        l_run[m] = T{};
#pragma unroll
        for (int w = 0; w < C::W; ++w) o[m][w] = V{};
    }
    bool ok = mbar_wait_bounded(bar0, 0);
    __syncthreads();

    int abort_kt = n_kt;
    for (int kt = 0; kt < n_kt; ++kt) {
        int const s = kt & 1;
        ok = ok && mbar_wait_bounded(bar0 + 8 * (1 + s), (kt >> 1) & 1);
        if (__syncthreads_or(!ok)) {
            ok = false;
            abort_kt = kt;
            break;
        }
        T const* Kt = Ks + s * C::TILE_ELEMS;
        T const* Vt = Vs + s * C::TILE_ELEMS;
        int64_t const key0 = static_cast<int64_t>(kt) * kBN;
        int const k_rows = static_cast<int>(min64(kBN, a.Tk - key0));
        // S = Q K^T for this thread's 4 x 4 block
        T sacc[4][C::KN];
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
            for (int n = 0; n < C::KN; ++n) sacc[m][n] = T{};
#pragma unroll 4
        for (int d0 = 0; d0 < D; d0 += C::NV) {
            V qv[4], kv[C::KN];
#pragma unroll
            for (int m = 0; m < 4; ++m) qv[m] = *reinterpret_cast<V const*>(Qs + (ty + 16 * m) * C::LD + d0);
#pragma unroll
            for (int n = 0; n < C::KN; ++n) kv[n] = *reinterpret_cast<V const*>(Kt + (tx + 16 * n) * C::LD + d0);
#pragma unroll
            for (int m = 0; m < 4; ++m)
#pragma unroll
                for (int n = 0; n < C::KN; ++n) sacc[m][n] = dotv<T>(qv[m], kv[n], sacc[m][n]);
        }

        // scale, mask, online softmax over this tile
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            int64_t const qi = q0 + ty + 16 * m;
            bool live[C::KN];
            T tmax = Lowest<T>::value;
#pragma unroll
            for (int n = 0; n < C::KN; ++n) {
                int64_t const kj = key0 + tx + 16 * n;
                live[n] = kj < a.Tk && !(a.causal && qi < kj);
                sacc[m][n] = sacc[m][n] * scale;  // attentionScores, then ops::scale
                if (live[n]) tmax = fmax(tmax, sacc[m][n]);
            }
            T const m_new = fmax(m_run[m], half_max(tmax));
            T const alpha = exp_t(m_run[m] - m_new);
            T psum{};
#pragma unroll
            for (int n = 0; n < C::KN; ++n) {
                T const p = live[n] ? exp_t(sacc[m][n] - m_new) : T{};
                Ps[(ty + 16 * m) * C::LDP + tx + 16 * n] = p;
                psum += p;
            }
            l_run[m] = l_run[m] * alpha + half_sum(psum);
            m_run[m] = m_new;
#pragma unroll
            for (int w = 0; w < C::W; ++w) {
                if constexpr (C::NV == 4) {
                    o[m][w].x *= alpha; o[m][w].y *= alpha; o[m][w].z *= alpha; o[m][w].w *= alpha;
                } else {
                    o[m][w].x *= alpha; o[m][w].y *= alpha;
                }
            }
        }
        __syncthreads();

        // O += P V
        int const kmax = min(kBN, k_rows);
#pragma unroll 4
        for (int j = 0; j < kmax; ++j) {
            T pv[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) pv[m] = Ps[(ty + 16 * m) * C::LDP + j];
#pragma unroll
            for (int w = 0; w < C::W; ++w) {
                V const vv = *reinterpret_cast<V const*>(Vt + j * C::LD + (tx + 16 * w) * C::NV);
#pragma unroll
                for (int m = 0; m < 4; ++m) axpyv<T>(o[m][w], pv[m], vv);
            }
        }
        __syncthreads();
        if (warp == 0 && kt + 2 < n_kt) issue_kv(kt + 2);
    }

    if (!ok) {
        if (tid == 0) {
            atomicOr(&g_prefill_error, ANN_DEVERR_WAIT_TIMEOUT);
            for (int t = abort_kt; t < min(n_kt, abort_kt + 2); ++t)  // drain copies in flight (bounded)
                mbar_wait_bounded(bar0 + 8 * (1 + (t & 1)), (t >> 1) & 1);
        }
        return;
    }
    T* obase = static_cast<T*>(a.out) + b * a.o_b + q0 * a.o_t + hq * a.o_h;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        int const r = ty + 16 * m;
        if (r >= q_rows) continue;
        T const l = l_run[m];
        T* orow = obase + r * a.o_t;
#pragma unroll
        for (int w = 0; w < C::W; ++w) {
            int const d = (tx + 16 * w) * C::NV;
            T vals[C::NV];
            if constexpr (C::NV == 4) {
                vals[0] = o[m][w].x; vals[1] = o[m][w].y; vals[2] = o[m][w].z; vals[3] = o[m][w].w;
            } else {
                vals[0] = o[m][w].x; vals[1] = o[m][w].y;
            }
#pragma unroll
            for (int e = 0; e < C::NV; ++e) orow[(d + e) * a.o_d] = l > T{} ? vals[e] / l : T{};
        }
    }
}

template <typename T, int D, int BN>
int launch(ann_stream stream, PrefillArgs& a, T scale, int64_t batch_heads) {
    using C = PCfg<T, D, BN>;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(prefill_kernel<T, D, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(C::SMEM));
    });
    if (attr != cudaSuccess) return fail(ANN_ECUDA, "attention prefill setup: %s", cudaGetErrorString(attr));
    int64_t const q_tiles = ceil_div(a.Tq, kBM);
    if (q_tiles * batch_heads > INT32_MAX)
        return fail(ANN_ENOTSUP, "attention prefill: grid too large for this build.");
    a.q_tiles = static_cast<int>(q_tiles);
    a.bhs = batch_heads;
    a.head_chunk = head_chunk_for(batch_heads, q_tiles, 2 * a.Tk * D * static_cast<int64_t>(sizeof(T)), 1);
    dim3 grid(static_cast<unsigned>(q_tiles * batch_heads));
    prefill_kernel<T, D, BN><<<grid, kThreads, C::SMEM, as_stream(stream)>>>(a, scale);
    return check_launch("attention prefill");
}

template <typename T>
int prefill(ann_stream stream, const ann_view* q_v, const ann_view* k_v, const ann_view* v_v, const ann_view* o_v,
            T scale, uint32_t g, int layout, int causal, void* mirror = nullptr) {
    if (g == 0u) return fail(ANN_EINVAL, "attention prefill requires queriesPerKvGroup > 0.");
    if (layout != ANN_LAYOUT_BTHD && layout != ANN_LAYOUT_BHTD)
        return fail(ANN_EINVAL, "attention prefill: invalid kv layout.");
    Dims q, k, v, o;
    ANN_TRY(to_dims(q_v, sizeof(T), "attention prefill Q", q));
    ANN_TRY(to_dims(k_v, sizeof(T), "attention prefill K", k));
    ANN_TRY(to_dims(v_v, sizeof(T), "attention prefill V", v));
    ANN_TRY(to_dims(o_v, sizeof(T), "attention prefill out", o));
    if (q.rank != 4 || k.rank != 4 || v.rank != 4 || o.rank != 4)
        return fail(ANN_EINVAL, "attention prefill expects rank-4 tensors.");
    if (!same_extents(q, o)) return fail(ANN_EINVAL, "attention prefill: out must have the extents of Q.");
    if (!same_extents(k, v)) return fail(ANN_EINVAL, "attention prefill: K and V extents differ.");
    int const tok = layout == ANN_LAYOUT_BTHD ? 1 : 2, head = layout == ANN_LAYOUT_BTHD ? 2 : 1;
    int64_t const B = q.ext[0], Tq = q.ext[1], Hq = q.ext[2], D = q.ext[3];
    if (k.ext[0] != B || k.ext[3] != D || k.ext[head] <= (Hq - 1) / static_cast<int64_t>(g))
        return fail(ANN_EINVAL, "attention prefill: Q %s does not match K/V %s.", extents_str(q).c_str(),
                    extents_str(k).c_str());
    if (q.numel() == 0) return ANN_OK;
    if (D != 64 && D != 128)
        return fail(ANN_ENOTSUP, "attention prefill: head dim %lld not supported.", static_cast<long long>(D));
    size_t const eb = sizeof(T);
    bool const unit = q.str[3] == 1 && k.str[3] == 1 && v.str[3] == 1;
    bool al = aligned(q.data, 16) && aligned(k.data, 16) && aligned(v.data, 16);
    for (int i = 0; i < 3; ++i)
        al = al && (q.str[i] * eb) % 16 == 0 && (k.str[i] * eb) % 16 == 0 && (v.str[i] * eb) % 16 == 0;
    if (!unit || !al)
        return fail(ANN_ENOTSUP, "attention prefill needs unit-stride head vectors and 16-byte aligned rows.");
    {  // fp32: tcgen05 3xTF32 kernel on SM pairs, else on single SMs; fp64: FP64 tensor-core (DMMA) kernel
        bool handled = false;
        int rc;
        if (mirror != nullptr && !aligned(mirror, sizeof(T)))
            return fail(ANN_EINVAL, "attention prefill: the output mirror is misaligned.");
        if constexpr (sizeof(T) == 4) {
            rc = ANN_OK;
            if (mirror || !std::getenv("ANN_PREFILL_FMA") || std::getenv("ANN_PREFILL_FMA")[0] != '1')
                rc = prefill_tc_pair_f32(stream, q, k, v, o, scale, g, layout, causal ? 1 : 0, handled, mirror);
            if (!handled && rc == ANN_OK && mirror == nullptr)
                rc = prefill_tc_f32(stream, q, k, v, o, scale, g, layout, causal ? 1 : 0, handled);
        } else
            rc = prefill_mma_f64(stream, q, k, v, o, scale, g, layout, causal ? 1 : 0, handled, mirror);
        if (handled || rc != ANN_OK) return rc;
        if (mirror != nullptr)
            return fail(ANN_ENOTSUP, "attention prefill: the multicast output needs the tensor-core kernels "
                                     "(head dim 64 or 128).");
    }
    PrefillArgs a{};
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
    a.Tk = k.ext[tok];
    a.Hq = Hq;
    a.g = g;
    a.causal = causal ? 1 : 0;
    if (D == 64) return launch<T, 64, 64>(stream, a, scale, B * Hq);
    // fp64 rows of 128 are 1 KB: 32-key tiles keep Q, two K/V stages and P within shared memory
    return launch<T, 128, (sizeof(T) == 8 ? 32 : 64)>(stream, a, scale, B * Hq);
}

}  // namespace

int take_prefill_error(cudaStream_t s, uint32_t* bits) {
    unsigned int value = 0, zero = 0;
    if (cudaMemcpyFromSymbolAsync(&value, g_prefill_error, sizeof value, 0, cudaMemcpyDeviceToHost, s) !=
            cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_prefill_error, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ANN_ECUDA, "device error word: %s", cudaGetErrorString(cudaGetLastError()));
    *bits |= value;
    return ANN_OK;
}

}  // namespace ann

extern "C" {

int ann_attention_prefill_f32(ann_stream s, const ann_view* q, const ann_view* k, const ann_view* v,
                              const ann_view* out, float scale, uint32_t g, int32_t layout, int32_t causal) {
    ANN_API_BEGIN
    return ann::prefill<float>(s, q, k, v, out, scale, g, layout, causal);
    ANN_API_END
}

int ann_attention_prefill_f64(ann_stream s, const ann_view* q, const ann_view* k, const ann_view* v,
                              const ann_view* out, double scale, uint32_t g, int32_t layout, int32_t causal) {
    ANN_API_BEGIN
    return ann::prefill<double>(s, q, k, v, out, scale, g, layout, causal);
    ANN_API_END
}

int ann_attention_prefill_mirror_f32(ann_stream s, const ann_view* q, const ann_view* k, const ann_view* v,
                                     const ann_view* out, void* out_mirror, float scale, uint32_t g, int32_t layout,
                                     int32_t causal) {
    ANN_API_BEGIN
    if (out_mirror == nullptr) return ann::fail(ANN_EINVAL, "attention prefill: the output mirror is NULL.");
    return ann::prefill<float>(s, q, k, v, out, scale, g, layout, causal, out_mirror);
    ANN_API_END
}

int ann_attention_prefill_mirror_f64(ann_stream s, const ann_view* q, const ann_view* k, const ann_view* v,
                                     const ann_view* out, void* out_mirror, double scale, uint32_t g,
                                     int32_t layout, int32_t causal) {
    ANN_API_BEGIN
    if (out_mirror == nullptr) return ann::fail(ANN_EINVAL, "attention prefill: the output mirror is NULL.");
    return ann::prefill<double>(s, q, k, v, out, scale, g, layout, causal, out_mirror);
    ANN_API_END
}

}  // extern "C"
