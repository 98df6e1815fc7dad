// prefill_tc.cu -- fp32 fused prefill attention on the sm_100a tensor cores (tcgen05), 3xTF32.
//
// Same pipeline and semantics as prefill.cu (attentionScores -> ops::scale ->
// causalSoftmax with the top-left mask / softmax -> attentionApply, reference
// test/unit/nn/attention.cpp:591-651), with both contractions on tcgen05.mma
// kind::tf32 and fp32 accuracy kept by the 3xTF32 split: every fp32 operand x
// is stored as hi = tf32(x) and lo = x - hi, and each product uses
// hi*hi + hi*lo + lo*hi (the dropped lo*lo term is ~2^-22 relative).
//
// One CTA (4 warps, one query row per thread = one TMEM lane) owns 128 query
// rows of one (batch, head):
//   TMEM  [Q_hi | Q_lo | S (32) | P_hi (32) | P_lo (32) | O (D)]   <= 480 of 512 columns
//   smem  raw K/V tiles of 32 keys, two stages, written by 4-D TMA in the
//         layouts the MMA reads (K: 128-byte swizzle, 16-byte chunks, K-major;
//         V: 128-byte swizzle, 32-byte chunks, MN-major); split once into
//         K_hi/K_lo/V_hi/V_lo with the same layouts
// Per key tile:
//   K raw -> split -> S = Q K^T      (A = Q from TMEM, B = K K-major, N = 32)
//   V raw -> split (overlaps the S MMAs)
//   S -> registers (tcgen05.ld): scale, top-left mask, online softmax with a
//        lazy rescale (O and l are rescaled only when the running max grows by
//        more than 8, exact because O and l share the reference max)
//   P_hi, P_lo -> TMEM (tcgen05.st);  O += P V   (A = P from TMEM, B = V MN-major)
// MMAs are issued by one thread and complete on mbarriers (tcgen05.commit);
// every wait is bounded, and on a timeout the CTA drains, frees its TMEM and
// reports ANN_DEVERR_WAIT_TIMEOUT.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "reduce.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace ann {

int prefill_tc_f32(ann_stream stream, const Dims& q, const Dims& k, const Dims& v, const Dims& o, float scale,
                   uint32_t g, int layout, int causal, bool& handled);
int take_prefill_tc_error(cudaStream_t s, uint32_t* bits);

namespace {

__device__ unsigned int g_tc_error;

constexpr int kBM = 128, kBN = 32, kThreads = 128;
constexpr float kLazy = 8.0f;  // rescale O only when the running max grows by more than this

template <int D>
struct TcCfg {
    static constexpr int TILE = kBN * D * 4;  // bytes of one K or V tile
    static constexpr int OFF_RAWK = 0;        // 2 stages
    static constexpr int OFF_RAWV = 2 * TILE;  // 2 stages
    static constexpr int OFF_KHI = 4 * TILE;
    static constexpr int OFF_KLO = 5 * TILE;
    static constexpr int OFF_VHI = 6 * TILE;
    static constexpr int OFF_VLO = 7 * TILE;
    static constexpr int OFF_BAR = 8 * TILE;  // barK[2], barV[2], barS, barPV
    static constexpr int OFF_SLOT = OFF_BAR + 6 * 8;
    static constexpr int USED = OFF_SLOT + 16;
    // + 1 KB for aligning the base to the 1 KB swizzle atom; at least 120 KB so
    // that a single CTA is resident per SM (it allocates all 512 TMEM columns)
    static constexpr int SMEM = USED + 1024 > 120 * 1024 ? USED + 1024 : 120 * 1024;
    static constexpr uint32_t Q_HI = 0, Q_LO = D, S_COL = 2 * D, P_HI = 2 * D + 32, P_LO = 2 * D + 64,
                              O_COL = 2 * D + 96;
    static constexpr uint32_t TMEM_COLS = 512;
    static_assert(O_COL + D <= TMEM_COLS, "TMEM budget");
    static constexpr uint32_t IDESC_S = tc::idesc_tf32(kBM, kBN, false);
    static constexpr uint32_t IDESC_PV = tc::idesc_tf32(kBM, D, true);
};

struct TcArgs {
    void* out;
    const float* q;
    int64_t q_b, q_t, q_h;
    int64_t o_b, o_t, o_h, o_d;
    int64_t Tq, Tk, Hq;
    uint32_t g;
    int causal;
    int kv_bthd;  // tensor-map coordinate order: 1 = (d, head, token, batch), 0 = (d, token, head, batch)
    int q_tiles;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, TcArgs a,
                      float scale) {
    using C = TcCfg<D>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    uint32_t const raw_base = smem_u32(smem_raw);
    uint32_t const pad = (1024u - (raw_base & 1023u)) & 1023u;
    unsigned char* smem = smem_raw + pad;
    uint32_t const sbase = raw_base + pad;
    uint32_t const barK0 = sbase + C::OFF_BAR, barV0 = barK0 + 16, barS = barK0 + 32, barPV = barK0 + 40;
    uint32_t* slot = reinterpret_cast<uint32_t*>(smem + C::OFF_SLOT);

    int const tid = threadIdx.x, warp = tid >> 5;
    int const qt = a.q_tiles - 1 - static_cast<int>(blockIdx.x);
    int64_t const bh = blockIdx.y;
    int64_t const hq = bh % a.Hq, b = bh / a.Hq, kvh = hq / a.g;
    int64_t const q0 = static_cast<int64_t>(qt) * kBM;
    int64_t const qi = q0 + tid;  // this thread's query row
    int64_t const k_end = a.causal ? (a.Tk < q0 + kBM ? a.Tk : q0 + kBM) : a.Tk;
    int const n_kt = static_cast<int>((k_end + kBN - 1) / kBN);

    if (tid == 0) {
        for (int i = 0; i < 6; ++i) mbar_init(barK0 + 8 * i, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(smem_u32(slot), C::TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    uint32_t const tmem = *slot;
    uint32_t const lane_off = static_cast<uint32_t>(warp * 32) << 16;

    auto issue_tile = [&](CUtensorMap const* map, uint32_t dst, uint32_t bar, int kt) {
        mbar_arrive_expect_tx(bar, C::TILE);
        int const t0 = kt * kBN;
        for (int blk = 0; blk < D / 32; ++blk) {
            uint32_t const d = dst + blk * (kBN * 128);
            if (a.kv_bthd)
                tc::tma_load_4d(d, map, blk * 32, static_cast<int>(kvh), t0, static_cast<int>(b), bar);
            else
                tc::tma_load_4d(d, map, blk * 32, t0, static_cast<int>(kvh), static_cast<int>(b), bar);
        }
    };
    if (tid == 0) {
        for (int kt = 0; kt < (n_kt < 2 ? n_kt : 2); ++kt) {
            issue_tile(&kmap, sbase + C::OFF_RAWK + kt * C::TILE, barK0 + 8 * kt, kt);
            issue_tile(&vmap, sbase + C::OFF_RAWV + kt * C::TILE, barV0 + 8 * kt, kt);
        }
    }

    // Q row -> TMEM as hi / lo (A operand of S = Q K^T)
    {
        float const* qrow = a.q + b * a.q_b + qi * a.q_t + hq * a.q_h;
        bool const live = qi < a.Tq;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
            float hi[32], lo[32];
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                float4 const x = live ? *reinterpret_cast<float4 const*>(qrow + 32 * c + j) : make_float4(0, 0, 0, 0);
                float const xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    hi[j + e] = tc::to_tf32(xs[e]);
                    lo[j + e] = xs[e] - hi[j + e];
                }
            }
            tc::tmem_st32(tmem + lane_off + C::Q_HI + 32 * c, hi);
            tc::tmem_st32(tmem + lane_off + C::Q_LO + 32 * c, lo);
        }
        tc::tmem_st_wait();
    }
    tc::fence_before_sync();
    __syncthreads();

    float m_used = Lowest<float>::value, l_sum = 0.f;
    bool ok = true;
    int pending_s = 0, pending_pv = 0;  // MMA groups issued and not yet waited (thread 0 tracks)
    int waited_k = 0, waited_v = 0;     // TMA tiles waited so far

    auto split_tile = [&](int raw_off, int hi_off, int lo_off) {
        float4 const* raw = reinterpret_cast<float4 const*>(smem + raw_off);
        float4* hi = reinterpret_cast<float4*>(smem + hi_off);
        float4* lo = reinterpret_cast<float4*>(smem + lo_off);
#pragma unroll 4
        for (int i = tid; i < C::TILE / 16; i += kThreads) {
            float4 const x = raw[i];
            float4 h, l;
            h.x = tc::to_tf32(x.x); h.y = tc::to_tf32(x.y); h.z = tc::to_tf32(x.z); h.w = tc::to_tf32(x.w);
            l.x = x.x - h.x; l.y = x.y - h.y; l.z = x.z - h.z; l.w = x.w - h.w;
            hi[i] = h;
            lo[i] = l;
        }
        tc::fence_proxy_async_smem();
    };

    for (int t = 0; t < n_kt; ++t) {
        int const s = t & 1;
        uint32_t const par = (t >> 1) & 1;
        // ---- K tile -> S = Q K^T -------------------------------------------------
        ok = mbar_wait_bounded(barK0 + 8 * s, par);
        if (__syncthreads_or(!ok)) break;
        waited_k = t + 1;
        split_tile(C::OFF_RAWK + s * C::TILE, C::OFF_KHI, C::OFF_KLO);
        __syncthreads();
        if (tid == 0) {
            if (t + 2 < n_kt) issue_tile(&kmap, sbase + C::OFF_RAWK + s * C::TILE, barK0 + 8 * s, t + 2);
            tc::fence_after_sync();
#pragma unroll 1
            for (int kk = 0; kk < D / 8; ++kk) {
                uint32_t const boff = (kk >> 2) * (kBN * 128) + (kk & 3) * 32;
                uint64_t const khi = tc::smem_desc(sbase + C::OFF_KHI + boff, 16, 1024, tc::kSwizzle128B);
                uint64_t const klo = tc::smem_desc(sbase + C::OFF_KLO + boff, 16, 1024, tc::kSwizzle128B);
                uint32_t const d = tmem + C::S_COL;
                tc::mma_tf32_ts(d, tmem + C::Q_HI + 8 * kk, khi, C::IDESC_S, kk > 0);
                tc::mma_tf32_ts(d, tmem + C::Q_HI + 8 * kk, klo, C::IDESC_S, 1);
                tc::mma_tf32_ts(d, tmem + C::Q_LO + 8 * kk, khi, C::IDESC_S, 1);
            }
            tc::mma_commit(barS);
        }
        pending_s = 1;
        // ---- V tile split (overlaps the S MMAs); needs the previous P V done ------
        ok = mbar_wait_bounded(barV0 + 8 * s, par);
        if (ok && t > 0) ok = mbar_wait_bounded(barPV, (t - 1) & 1);
        if (__syncthreads_or(!ok)) break;
        waited_v = t + 1;
        pending_pv = 0;
        tc::fence_after_sync();
        split_tile(C::OFF_RAWV + s * C::TILE, C::OFF_VHI, C::OFF_VLO);
        // ---- softmax on S ------------------------------------------------------------
        ok = mbar_wait_bounded(barS, t & 1);
        if (__syncthreads_or(!ok)) break;
        pending_s = 0;
        tc::fence_after_sync();
        float sv[32];
        tc::tmem_ld32(tmem + lane_off + C::S_COL, sv);
        int64_t const key0 = static_cast<int64_t>(t) * kBN;
        float tmax = Lowest<float>::value;
        bool live[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            int64_t const kj = key0 + j;
            live[j] = kj < a.Tk && !(a.causal && qi < kj);
            sv[j] = sv[j] * scale;  // attentionScores, then ops::scale
            if (live[j]) tmax = fmaxf(tmax, sv[j]);
        }
        bool const grow = tmax > m_used + kLazy;
        float alpha = 1.f;
        if (grow) {
            alpha = expf(m_used - tmax);
            m_used = tmax;
            l_sum *= alpha;
        }
        if (t > 0 && __any_sync(0xffffffffu, grow)) {  // warp-uniform: tcgen05.ld/st are warp-collective
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                float ov[32];
                tc::tmem_ld32(tmem + lane_off + C::O_COL + 32 * c, ov);
#pragma unroll
                for (int j = 0; j < 32; ++j) ov[j] *= alpha;
                tc::tmem_st32(tmem + lane_off + C::O_COL + 32 * c, ov);
            }
        }
        float phi[32], plo[32], psum = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            float const p = live[j] ? expf(sv[j] - m_used) : 0.f;
            psum += p;
            phi[j] = tc::to_tf32(p);
            plo[j] = p - phi[j];
        }
        l_sum += psum;
        tc::tmem_st32(tmem + lane_off + C::P_HI, phi);
        tc::tmem_st32(tmem + lane_off + C::P_LO, plo);
        tc::tmem_st_wait();
        tc::fence_before_sync();
        __syncthreads();
        // ---- O += P V ------------------------------------------------------------------
        if (tid == 0) {
            if (t + 2 < n_kt) issue_tile(&vmap, sbase + C::OFF_RAWV + s * C::TILE, barV0 + 8 * s, t + 2);
            tc::fence_after_sync();
#pragma unroll 1
            for (int kk = 0; kk < kBN / 8; ++kk) {
                uint64_t const vhi = tc::smem_desc(sbase + C::OFF_VHI + kk * 1024, kBN * 128, 512, tc::kSwizzle128B_32B);
                uint64_t const vlo = tc::smem_desc(sbase + C::OFF_VLO + kk * 1024, kBN * 128, 512, tc::kSwizzle128B_32B);
                uint32_t const d = tmem + C::O_COL;
                tc::mma_tf32_ts(d, tmem + C::P_HI + 8 * kk, vhi, C::IDESC_PV, (t > 0 || kk > 0) ? 1u : 0u);
                tc::mma_tf32_ts(d, tmem + C::P_HI + 8 * kk, vlo, C::IDESC_PV, 1);
                tc::mma_tf32_ts(d, tmem + C::P_LO + 8 * kk, vhi, C::IDESC_PV, 1);
            }
            tc::mma_commit(barPV);
        }
        pending_pv = 1;
    }

    if (ok && n_kt > 0) {
        ok = mbar_wait_bounded(barPV, (n_kt - 1) & 1);
        ok = !__syncthreads_or(!ok);
        if (ok) pending_pv = 0;
    }
    if (ok) {
        tc::fence_after_sync();
        float* orow = static_cast<float*>(a.out) + b * a.o_b + qi * a.o_t + hq * a.o_h;
        float const inv_ok = l_sum > 0.f ? 1.f : 0.f;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
            float ov[32];
            tc::tmem_ld32(tmem + lane_off + C::O_COL + 32 * c, ov);
            if (qi < a.Tq) {
#pragma unroll
                for (int j = 0; j < 32; ++j) orow[(32 * c + j) * a.o_d] = inv_ok > 0.f ? ov[j] / l_sum : 0.f;
            }
        }
    } else if (tid == 0) {
        atomicOr(&g_tc_error, ANN_DEVERR_WAIT_TIMEOUT);
        // drain: copies and MMAs still in flight must land before the CTA leaves
        for (int t = waited_k; t < (n_kt < waited_k + 2 ? n_kt : waited_k + 2); ++t)
            mbar_wait_bounded(barK0 + 8 * (t & 1), (t >> 1) & 1);
        for (int t = waited_v; t < (n_kt < waited_v + 2 ? n_kt : waited_v + 2); ++t)
            mbar_wait_bounded(barV0 + 8 * (t & 1), (t >> 1) & 1);
        if (pending_s) mbar_wait_bounded(barS, (waited_k - 1) & 1);
        if (pending_pv) mbar_wait_bounded(barPV, (waited_v - 1) & 1);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 4-D map over K or V with dims ordered by increasing stride:
// BTHD (d, head, token, batch) or BHTD (d, token, head, batch); box = 32 d x 32 tokens.
bool make_kv_map(CUtensorMap& map, const Dims& t, int layout, CUtensorMapSwizzle swizzle) {
    auto enc = encode_fn();
    if (enc == nullptr) return false;
    int const tok = layout == ANN_LAYOUT_BTHD ? 1 : 2, head = layout == ANN_LAYOUT_BTHD ? 2 : 1;
    int const d1 = layout == ANN_LAYOUT_BTHD ? head : tok, d2 = layout == ANN_LAYOUT_BTHD ? tok : head;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(t.ext[3]), static_cast<cuuint64_t>(t.ext[d1]),
                          static_cast<cuuint64_t>(t.ext[d2]), static_cast<cuuint64_t>(t.ext[0])};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(t.str[d1]) * 4, static_cast<cuuint64_t>(t.str[d2]) * 4,
                             static_cast<cuuint64_t>(t.str[0]) * 4};
    // strides must grow with the dimension (each one covers the previous dimension)
    if (strides[0] < dims[0] * 4 || strides[1] < strides[0] * dims[1] || strides[2] < strides[1] * dims[2])
        return false;
    for (int i = 0; i < 4; ++i)
        if (dims[i] == 0) return false;
    cuuint32_t box[4] = {32, layout == ANN_LAYOUT_BTHD ? 1u : static_cast<cuuint32_t>(kBN),
                         layout == ANN_LAYOUT_BTHD ? static_cast<cuuint32_t>(kBN) : 1u, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult const r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, t.data, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int D>
int launch_tc(ann_stream stream, const Dims& q, const Dims& k, const Dims& v, const Dims& o, float scale, uint32_t g,
              int layout, int causal, bool& handled) {
    using C = TcCfg<D>;
    CUtensorMap kmap, vmap;
    // K is the K-major B operand of S = Q K^T (16-byte swizzle chunks); V is the
    // MN-major B operand of O = P V, which for 32-bit elements needs 32-byte chunks.
    if (!make_kv_map(kmap, k, layout, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_kv_map(vmap, v, layout, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
        return ANN_OK;  // not handled
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(prefill_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    if (attr != cudaSuccess) return fail(ANN_ECUDA, "attention prefill (tensor cores) setup: %s",
                                         cudaGetErrorString(attr));
    TcArgs a{};
    a.out = o.data;
    a.q = static_cast<const float*>(q.data);
    a.q_b = q.str[0];
    a.q_t = q.str[1];
    a.q_h = q.str[2];
    a.o_b = o.str[0];
    a.o_t = o.str[1];
    a.o_h = o.str[2];
    a.o_d = o.str[3];
    a.Tq = q.ext[1];
    a.Tk = layout == ANN_LAYOUT_BTHD ? k.ext[1] : k.ext[2];
    a.Hq = q.ext[2];
    a.g = g;
    a.causal = causal;
    a.kv_bthd = layout == ANN_LAYOUT_BTHD ? 1 : 0;
    int64_t const q_tiles = ceil_div(a.Tq, kBM);
    int64_t const bhs = q.ext[0] * q.ext[2];
    if (q_tiles > INT32_MAX || bhs > 65535) return ANN_OK;  // not handled
    a.q_tiles = static_cast<int>(q_tiles);
    handled = true;
    dim3 grid(static_cast<unsigned>(q_tiles), static_cast<unsigned>(bhs));
    prefill_tc_kernel<D><<<grid, kThreads, C::SMEM, as_stream(stream)>>>(kmap, vmap, a, scale);
    return check_launch("attention prefill (tensor cores)");
}

}  // namespace

// Runs the tensor-core kernel when the shapes allow it (fp32, D 64/128, a TMA
// map can describe K and V); sets `handled` = false otherwise.
int prefill_tc_f32(ann_stream stream, const Dims& q, const Dims& k, const Dims& v, const Dims& o, float scale,
                   uint32_t g, int layout, int causal, bool& handled) {
    handled = false;
    if (const char* env = std::getenv("ANN_PREFILL_FMA"))
        if (env[0] == '1') return ANN_OK;
    if (q.ext[3] == 64) return launch_tc<64>(stream, q, k, v, o, scale, g, layout, causal, handled);
    if (q.ext[3] == 128) return launch_tc<128>(stream, q, k, v, o, scale, g, layout, causal, handled);
    return ANN_OK;
}

int take_prefill_tc_error(cudaStream_t s, uint32_t* bits) {
    unsigned int value = 0, zero = 0;
    if (cudaMemcpyFromSymbolAsync(&value, g_tc_error, sizeof value, 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_tc_error, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ANN_ECUDA, "device error word: %s", cudaGetErrorString(cudaGetLastError()));
    *bits |= value;
    return ANN_OK;
}

}  // namespace ann
