// prefill_tc.cu -- fp32 fused prefill attention on the sm_100a tensor cores (tcgen05), 3xTF32.
//
// Same pipeline and semantics as prefill.cu (attentionScores -> ops::scale ->
// causalSoftmax with the top-left mask / softmax -> attentionApply, reference
// test/unit/nn/attention.cpp:591-651), with both contractions on tcgen05.mma
// kind::tf32 and fp32 accuracy kept by the 3xTF32 split: every fp32 operand x
// is stored as hi = tf32(x) and lo = x - hi, and each product uses
// hi*hi + hi*lo + lo*hi (the dropped lo*lo term is ~2^-22 relative).
//
// One CTA owns 128 query rows of one (batch, head): warps 0..3 hold one query
// row per thread (= one TMEM lane) and do the hi/lo splits and the softmax;
// warp 4 issues the TMA copies and the MMAs (warp specialisation, so the MMA
// issue stream never waits behind the softmax):
//   TMEM  [Q_hi | Q_lo | S (32) | P_hi (32) | P_lo (32) | O (D)]   <= 480 of 512 columns
//   smem  raw K/V tiles of 32 keys, kRaw stages each, written by 4-D TMA in the
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

constexpr int kBM = 128, kBN = 32;
constexpr int kRaw = 4;  // raw K / V stages (TMA prefetch depth in key tiles)
constexpr int kSoftmaxThreads = 128;                 // warps 0..3: one query row (TMEM lane) per thread
constexpr int kThreads = kSoftmaxThreads + 32;       // warp 4: TMA + MMA producer
constexpr float kLazy = 8.0f;  // rescale O only when the running max grows by more than this

template <int D>
struct TcCfg {
    static constexpr int TILE = kBN * D * 4;  // bytes of one K or V tile
    static constexpr int OFF_RAWK = 0;               // kRaw stages
    static constexpr int OFF_RAWV = kRaw * TILE;     // kRaw stages
    static constexpr int OFF_KHI = 2 * kRaw * TILE;
    static constexpr int OFF_KLO = OFF_KHI + TILE;
    static constexpr int OFF_VHI = OFF_KHI + 2 * TILE;
    static constexpr int OFF_VLO = OFF_KHI + 3 * TILE;
    static constexpr int OFF_BAR = OFF_KHI + 4 * TILE;
    // barriers: kfull[kRaw] vfull[kRaw] kready vready sfull[2] sfree[2] pfull pvdone
    static constexpr int NBAR = 2 * kRaw + 8;
    static constexpr int OFF_SLOT = OFF_BAR + NBAR * 8;  // TMEM base, abort flag, progress counters
    static constexpr int USED = OFF_SLOT + 32;
    // + 1 KB to align the base to the 1 KB swizzle atom; >= 120 KB so that a
    // single CTA is resident per SM (it allocates all 512 TMEM columns)
    static constexpr int SMEM = USED + 1024 > 120 * 1024 ? USED + 1024 : 120 * 1024;
    // TMEM columns: Q_hi | Q_lo | S[0] | S[1] | P_hi | P_lo | O
    static constexpr uint32_t Q_HI = 0, Q_LO = D, S_COL = 2 * D, P_HI = 2 * D + 2 * kBN, P_LO = 2 * D + 3 * kBN,
                              O_COL = 2 * D + 4 * kBN;
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

// Pipeline per key tile t (tensor pipe order S(0), S(1), PV(0), S(2), PV(1), ...):
//   producer : wait kready(t) -> TMA K(t+kRaw) -> [sfree(t-2)] -> S(t) = Q K^T -> commit sfull[t%2]
//              wait pfull(t-1), vready(t-1) -> O += P V (t-1) -> commit pvdone -> TMA V(t-1+kRaw)
//   softmax  : wait sfull(t) -> split K(t+1) -> kready      (lets S(t+1) start at once)
//              wait pvdone(t-1), vfull(t) -> split V(t) -> vready
//              S(t) -> registers -> sfree; scale, mask, online softmax, lazy O rescale
//              P_hi, P_lo -> TMEM -> pfull
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
    uint32_t const bar = sbase + C::OFF_BAR;
    uint32_t const kfull = bar, vfull = bar + 8 * kRaw, kready = bar + 16 * kRaw, vready = kready + 8,
                   sfull = kready + 16, sfree = kready + 32, pfull = kready + 48, pvdone = kready + 56;
    uint32_t* slot = reinterpret_cast<uint32_t*>(smem + C::OFF_SLOT);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + C::OFF_SLOT + 4);
    volatile int* prog = reinterpret_cast<volatile int*>(smem + C::OFF_SLOT + 8);  // [0] K issued [1] V issued
                                                                                 // [2] K waited [3] V waited
                                                                                 // [4] last commit: 1 + 2*group

    int const tid = threadIdx.x, warp = tid >> 5;
    int const qt = a.q_tiles - 1 - static_cast<int>(blockIdx.x);
    int64_t const bh = blockIdx.y;
    int64_t const hq = bh % a.Hq, b = bh / a.Hq, kvh = hq / a.g;
    int64_t const q0 = static_cast<int64_t>(qt) * kBM;
    int64_t const k_end = a.causal ? (a.Tk < q0 + kBM ? a.Tk : q0 + kBM) : a.Tk;
    int const n_kt = static_cast<int>((k_end + kBN - 1) / kBN);

    if (tid == 0) {
        for (int i = 0; i < 2 * kRaw; ++i) mbar_init(bar + 8 * i, 1);  // kfull, vfull
        mbar_init(kready, kSoftmaxThreads);
        mbar_init(vready, kSoftmaxThreads);
        for (int i = 0; i < 2; ++i) mbar_init(sfull + 8 * i, 1);
        for (int i = 0; i < 2; ++i) mbar_init(sfree + 8 * i, kSoftmaxThreads);
        mbar_init(pfull, kSoftmaxThreads);
        mbar_init(pvdone, 1);
        fence_mbar_init();
        *abort = 0;
        for (int i = 0; i < 5; ++i) prog[i] = 0;
    }
    if (warp == 0) {
        tc::tmem_alloc(smem_u32(slot), C::TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    uint32_t const tmem = *slot;

    if (warp == 4) {
        // ================================ producer ================================
        if ((tid & 31) == 0) {
            auto issue_tile = [&](CUtensorMap const* map, uint32_t dst, uint32_t b_, int kt) {
                mbar_arrive_expect_tx(b_, C::TILE);
                int const t0 = kt * kBN;
                for (int blk = 0; blk < D / 32; ++blk) {
                    uint32_t const d = dst + blk * (kBN * 128);
                    if (a.kv_bthd)
                        tc::tma_load_4d(d, map, blk * 32, static_cast<int>(kvh), t0, static_cast<int>(b), b_);
                    else
                        tc::tma_load_4d(d, map, blk * 32, t0, static_cast<int>(kvh), static_cast<int>(b), b_);
                }
            };
            auto issue_pv = [&](int t) {  // O += P V for tile t
                tc::fence_after_sync();
#pragma unroll 1
                for (int kk = 0; kk < kBN / 8; ++kk) {
                    uint64_t const vhi = tc::smem_desc(sbase + C::OFF_VHI + kk * 1024, kBN * 128, 512,
                                                       tc::kSwizzle128B_32B);
                    uint64_t const vlo = tc::smem_desc(sbase + C::OFF_VLO + kk * 1024, kBN * 128, 512,
                                                       tc::kSwizzle128B_32B);
                    uint32_t const d = tmem + C::O_COL;
                    tc::mma_tf32_ts(d, tmem + C::P_HI + 8 * kk, vhi, C::IDESC_PV, (t > 0 || kk > 0) ? 1u : 0u);
                    tc::mma_tf32_ts(d, tmem + C::P_HI + 8 * kk, vlo, C::IDESC_PV, 1);
                    tc::mma_tf32_ts(d, tmem + C::P_LO + 8 * kk, vhi, C::IDESC_PV, 1);
                }
                tc::mma_commit(pvdone);
                prog[4] = 2 + 2 * t;  // pvdone, phase t & 1
            };
            int const pre = n_kt < kRaw ? n_kt : kRaw;
            for (int kt = 0; kt < pre; ++kt) {
                issue_tile(&kmap, sbase + C::OFF_RAWK + kt * C::TILE, kfull + 8 * kt, kt);
                issue_tile(&vmap, sbase + C::OFF_RAWV + kt * C::TILE, vfull + 8 * kt, kt);
            }
            prog[0] = pre;
            prog[1] = pre;
            bool ok = true;
            for (int t = 0; t < n_kt && ok; ++t) {
                ok = mbar_wait_or_abort(kready, t & 1, abort);
                if (!ok) break;
                if (t + kRaw < n_kt) {  // split K(t) has consumed raw stage t % kRaw
                    int const st = t % kRaw;
                    issue_tile(&kmap, sbase + C::OFF_RAWK + st * C::TILE, kfull + 8 * st, t + kRaw);
                    prog[0] = t + kRaw + 1;
                }
                if (t >= 2) ok = mbar_wait_or_abort(sfree + 8 * (t & 1), ((t - 2) >> 1) & 1, abort);
                if (!ok) break;
                tc::fence_after_sync();
                uint32_t const d = tmem + C::S_COL + (t & 1) * kBN;
#pragma unroll 1
                for (int kk = 0; kk < D / 8; ++kk) {
                    uint32_t const boff = (kk >> 2) * (kBN * 128) + (kk & 3) * 32;
                    uint64_t const khi = tc::smem_desc(sbase + C::OFF_KHI + boff, 16, 1024, tc::kSwizzle128B);
                    uint64_t const klo = tc::smem_desc(sbase + C::OFF_KLO + boff, 16, 1024, tc::kSwizzle128B);
                    tc::mma_tf32_ts(d, tmem + C::Q_HI + 8 * kk, khi, C::IDESC_S, kk > 0);
                    tc::mma_tf32_ts(d, tmem + C::Q_HI + 8 * kk, klo, C::IDESC_S, 1);
                    tc::mma_tf32_ts(d, tmem + C::Q_LO + 8 * kk, khi, C::IDESC_S, 1);
                }
                tc::mma_commit(sfull + 8 * (t & 1));
                prog[4] = 1 + 2 * t;  // sfull[t & 1], phase (t >> 1) & 1
                if (t >= 1) {
                    ok = mbar_wait_or_abort(pfull, (t - 1) & 1, abort) &&
                         mbar_wait_or_abort(vready, (t - 1) & 1, abort);
                    if (!ok) break;
                    issue_pv(t - 1);
                    if (t - 1 + kRaw < n_kt) {  // split V(t-1) has consumed raw stage (t-1) % kRaw
                        int const st = (t - 1) % kRaw;
                        issue_tile(&vmap, sbase + C::OFF_RAWV + st * C::TILE, vfull + 8 * st, t - 1 + kRaw);
                        prog[1] = t + kRaw;
                    }
                }
            }
            if (ok && n_kt > 0) {
                ok = mbar_wait_or_abort(pfull, (n_kt - 1) & 1, abort) &&
                     mbar_wait_or_abort(vready, (n_kt - 1) & 1, abort);
                if (ok) issue_pv(n_kt - 1);
            }
        }
    } else {
        // ======================= softmax / split warps (0..3) =======================
        uint32_t const lane_off = static_cast<uint32_t>(warp * 32) << 16;
        int64_t const qi = q0 + tid;
        // Q row -> TMEM as hi / lo (A operand of S = Q K^T)
        {
            float const* qrow = a.q + b * a.q_b + qi * a.q_t + hq * a.q_h;
            bool const live = qi < a.Tq;
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                float hi[32], lo[32];
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    float4 const x =
                        live ? *reinterpret_cast<float4 const*>(qrow + 32 * c + j) : make_float4(0, 0, 0, 0);
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
            tc::fence_before_sync();
        }
        auto split = [&](int raw_off, int hi_off, int lo_off) {
            float4 const* raw = reinterpret_cast<float4 const*>(smem + raw_off);
            float4* hi = reinterpret_cast<float4*>(smem + hi_off);
            float4* lo = reinterpret_cast<float4*>(smem + lo_off);
#pragma unroll 4
            for (int i = tid; i < C::TILE / 16; i += kSoftmaxThreads) {
                float4 const x = raw[i];
                float4 h, l;
                h.x = tc::to_tf32(x.x); h.y = tc::to_tf32(x.y); h.z = tc::to_tf32(x.z); h.w = tc::to_tf32(x.w);
                l.x = x.x - h.x; l.y = x.y - h.y; l.z = x.z - h.z; l.w = x.w - h.w;
                hi[i] = h;
                lo[i] = l;
            }
            tc::fence_proxy_async_smem();  // make the split visible to the tensor core
        };
        // Decisions after a wait are made warp-uniform (__all_sync): the tcgen05.ld/st
        // that follow are warp-collective, so a warp must never split on an abort.
        auto split_k = [&](int t) {
            int const st = t % kRaw;
            bool const w = __all_sync(0xffffffffu, mbar_wait_or_abort(kfull + 8 * st, (t / kRaw) & 1, abort));
            if (w) {
                if (tid == 0) prog[2] = t + 1;
                split(C::OFF_RAWK + st * C::TILE, C::OFF_KHI, C::OFF_KLO);
            }
            mbar_arrive(kready);
            return w;
        };
        float m_used = Lowest<float>::value, l_sum = 0.f;
        bool ok = n_kt == 0 || split_k(0);
        for (int t = 0; t < n_kt && ok; ++t) {
            ok = __all_sync(0xffffffffu, mbar_wait_or_abort(sfull + 8 * (t & 1), (t >> 1) & 1, abort));
            if (!ok) break;  // S(t) done: K_hi/K_lo free
            tc::fence_after_sync();
            if (t + 1 < n_kt && !split_k(t + 1)) {
                ok = false;
                break;
            }
            ok = (t == 0 || mbar_wait_or_abort(pvdone, (t - 1) & 1, abort)) &&
                 mbar_wait_or_abort(vfull + 8 * (t % kRaw), (t / kRaw) & 1, abort);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc::fence_after_sync();
            if (tid == 0) prog[3] = t + 1;
            split(C::OFF_RAWV + (t % kRaw) * C::TILE, C::OFF_VHI, C::OFF_VLO);
            mbar_arrive(vready);

            float sv[32];
            tc::tmem_ld32(tmem + lane_off + C::S_COL + (t & 1) * kBN, sv);
            tc::fence_before_sync();
            mbar_arrive(sfree + 8 * (t & 1));
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
            mbar_arrive(pfull);
        }
        if (ok && n_kt > 0) ok = mbar_wait_or_abort(pvdone, (n_kt - 1) & 1, abort);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
            tc::fence_after_sync();
            float* orow = static_cast<float*>(a.out) + b * a.o_b + qi * a.o_t + hq * a.o_h;
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                float ov[32];
                tc::tmem_ld32(tmem + lane_off + C::O_COL + 32 * c, ov);
                if (qi < a.Tq) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) orow[(32 * c + j) * a.o_d] = l_sum > 0.f ? ov[j] / l_sum : 0.f;
                }
            }
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (*abort && tid == kSoftmaxThreads) {
        // A wait gave up: drain the copies and MMAs still in flight before the TMEM goes.
        atomicOr(&g_tc_error, ANN_DEVERR_WAIT_TIMEOUT);
        for (int t = prog[2]; t < prog[0]; ++t) mbar_wait_bounded(kfull + 8 * (t % kRaw), (t / kRaw) & 1);
        for (int t = prog[3]; t < prog[1]; ++t) mbar_wait_bounded(vfull + 8 * (t % kRaw), (t / kRaw) & 1);
        int const last = prog[4];
        if (last > 0) {
            int const g = (last - 1) >> 1;
            if ((last & 1) == 1)
                mbar_wait_bounded(sfull + 8 * (g & 1), (g >> 1) & 1);
            else
                mbar_wait_bounded(pvdone, g & 1);
        }
    }
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
