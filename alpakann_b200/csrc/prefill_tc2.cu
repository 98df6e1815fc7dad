// prefill_tc2.cu -- fp32 fused prefill attention on pairs of SMs (tcgen05 cta_group::2), 3xTF32.
//
// The pipeline, semantics and per-row softmax of prefill_tc.cu (attentionScores
// -> ops::scale -> causalSoftmax with the top-left mask / softmax ->
// attentionApply, reference test/unit/nn/attention.cpp:591-651), on a cluster of
// two CTAs that share every MMA:
//   - a 256-row query tile per pair, CTA r holding rows [128 r, 128 r + 128);
//     one thread of CTA 0 issues M = 256 MMAs (cta_group::2) for both;
//   - CTA r stores keys [32 r, 32 r + 32) of each 64-key K tile and head dims
//     [D r / 2, D r / 2 + D / 2) of each V tile, so each SM writes and its
//     tensor core reads half of K and V per tile;
//   - the shared memory this frees holds Q_lo (the S MMA that needs it reads A
//     from shared memory), and the TMEM that frees holds two S accumulators:
//     S(t+1) is computed while the softmax of tile t still reads S(t).
// 3xTF32 as in prefill_tc.cu: x = hi + lo with hi the raw fp32 value (the MMA
// reads it as tf32) and lo = x - trunc13(x); S = Q_hi K_hi + Q_hi K_lo + Q_lo K_hi
// and O += P_hi V_hi + P_hi V_lo + P_lo V_hi.
//   TMEM  [Q_hi | O | S0 (64) | S1 (64) | P_hi (64)]            (D = 128: 448 columns)
//   smem  K hi/lo x 2 | V hi/lo x 2 (half tiles) | P_lo | Q_lo  (D = 128: 224 KB)
// Raw K and V tiles arrive by TMA tensor loads straight into the K_hi / V_hi
// buffers (a box is one column block of the K-major 128-byte-swizzled K layout
// or of the MN-major 32-byte-atom V layout); the row threads add the lo parts
// beside them. Q passes through the row threads' registers (Q_hi goes to TMEM).
// Row threads signal the barriers CTA 0's issuers wait on through the cluster
// window; the issuers commit each group of MMAs to both CTAs' barriers. Every
// wait is bounded; on a timeout both CTAs stop, the issuers drain their MMAs,
// both meet at a cluster barrier, free TMEM and report ANN_DEVERR_WAIT_TIMEOUT.
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "multimem.cuh"
#include "reduce.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"
#include "tmap.cuh"

namespace ann {

int prefill_tc_pair_f32(ann_stream stream, const Dims& q, const Dims& k, const Dims& v, const Dims& o, float scale,
                        uint32_t g, int layout, int causal, bool& handled, void* mirror);
int take_prefill_tc2_error(cudaStream_t s, uint32_t* bits);

namespace {

__device__ unsigned int g_tc2_error;

constexpr int kBM = 128, kBN = 64;  // rows per CTA, keys per tile
constexpr int kRowThreads = 256;    // warps 0..7
constexpr int kThreads = kRowThreads + 64;  // + warp 8 (S issuer) and warp 9 (PV issuer)
constexpr float kLog2e = 1.44269504088896341f;
constexpr float kLazy2 = 8.0f * kLog2e;  // lazy-rescale threshold, log2 units

template <int D>
struct PairCfg {
    static constexpr int KROWS = kBN / 2;            // keys of a K tile held by this CTA
    static constexpr int VCOLS = D / 2;              // head dims of a V tile held by this CTA
    static constexpr int TILE_K = KROWS * D * 4;     // bytes of K hi (or lo) per buffer
    static constexpr int TILE_V = kBN * VCOLS * 4;   // bytes of V hi (or lo)
    static constexpr int BLK_K = KROWS * 128;        // one 32-float column block of K
    static constexpr int BLK_V = kBN * 128;          // one 32-float column block of V
    static constexpr int PLO_BLK = kBM * 128;        // one 32-key column block of P_lo
    static constexpr int QLO_BLK = kBM * 128;        // one 32-dim column block of Q_lo
    static constexpr int OFF_K = 0;                  // buffer i: hi at OFF_K + 2*i*TILE_K, lo at + TILE_K
    static constexpr int OFF_V = 4 * TILE_K;         // buffer i: hi at OFF_V + 2*i*TILE_V, lo at + TILE_V
    static constexpr int OFF_PLO = OFF_V + 4 * TILE_V;
    static constexpr int OFF_QLO = OFF_PLO + 2 * PLO_BLK;
    static constexpr int OFF_BAR = OFF_QLO + (D / 32) * QLO_BLK;
    // barriers: qready kready[2] vready[2] sfull[2] sfree[2] pfull pvdone drain_s drain_pv kfull[2] vfull[2]
    static constexpr int NBAR = 17;
    static constexpr int OFF_SLOT = OFF_BAR + NBAR * 8;  // TMEM base, abort flag
    static constexpr int USED = OFF_SLOT + 16;
    // + 1 KB to align the base to the 1 KB swizzle atom; >= 120 KB so that a
    // single CTA is resident per SM (it allocates all 512 TMEM columns)
    static constexpr int SMEM = USED + 1024 > 120 * 1024 ? USED + 1024 : 120 * 1024;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static constexpr uint32_t Q_HI = 0, O_COL = D, S_COL = 2 * D, P_HI = 2 * D + 2 * kBN;  // S buffer b at S_COL + 64 b
    static constexpr uint32_t TMEM_COLS = 512;
    static_assert(P_HI + kBN <= TMEM_COLS, "TMEM budget");
    static constexpr uint32_t IDESC_S = tc::idesc_tf32(2 * kBM, kBN, false);
    static constexpr uint32_t IDESC_PV = tc::idesc_tf32(2 * kBM, D, true);
    static constexpr uint32_t ROW_ARRIVALS = 2 * kRowThreads;  // row threads of both CTAs
};

struct PairArgs {
    void* out;
    float* mirror;  // multicast address of out[0] (every O store goes to all ranks' copies), or null
    const float* q;
    const float* k;
    const float* v;
    int64_t q_b, q_t, q_h;
    int64_t k_b, k_t, k_h;
    int64_t v_b, v_t, v_h;
    int64_t o_b, o_t, o_h, o_d;
    int64_t Tq, Tk, Hq;
    uint32_t g;
    int causal;
    int o_vec;           // out rows are unit-stride and 16-byte aligned
    int q_tiles;         // 256-row tiles
    int64_t bhs;         // batch * query heads
    int64_t head_chunk;  // (batch, head) pairs per dispatch chunk
    int alternate;       // query tiles in the order heaviest, lightest, 2nd heaviest, ... (see launch_pair)
};

// lo part of the 3xTF32 split (see prefill_tc.cu): x - trunc13(x), exact in fp32.
__device__ __forceinline__ float tf32_lo(float x) {
    return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}
__device__ __forceinline__ float4 tf32_lo(float4 x) {
    return make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
}

// 2^x by the ex2.approx instruction (+0 for x = -inf or below -126)
__device__ __forceinline__ float exp2_approx(float x) {
    float p;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(p) : "f"(x));
    return p;
}

__device__ __forceinline__ void row_sync() {  // the 256 row threads (warps 0..7) of this CTA
    asm volatile("bar.sync 1, %0;" ::"n"(kRowThreads) : "memory");
}
// row_sync that also ORs `v` over the 256 row threads: every one gets the same answer
__device__ __forceinline__ bool row_sync_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v)), "n"(kRowThreads)
        : "memory");
    return r != 0;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1) prefill_pair_kernel(PairArgs a, float scale,
                                                                   const __grid_constant__ CUtensorMap kmap,
                                                                   const __grid_constant__ CUtensorMap vmap) {
    using C = PairCfg<D>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    uint32_t const raw_base = smem_u32(smem_raw);
    uint32_t const pad = (1024u - (raw_base & 1023u)) & 1023u;
    unsigned char* smem = smem_raw + pad;
    uint32_t const sbase = raw_base + pad;
    uint32_t const bar = sbase + C::OFF_BAR;
    uint32_t const qready = bar, kready = bar + 8, vready = bar + 24, sfull = bar + 40, sfree = bar + 56,
                   pfull = bar + 72, pvdone = bar + 80, drain_s = bar + 88, drain_pv = bar + 96, kfull = bar + 104,
                   vfull = bar + 120;
    uint32_t* slot = reinterpret_cast<uint32_t*>(smem + C::OFF_SLOT);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + C::OFF_SLOT + 4);

    int const tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int const rank = static_cast<int>(cluster_ctarank());
    // 1-D grid of pairs in chunks of a.head_chunk (batch, head) pairs
    // (head_chunk_for): inside a chunk the query tiles go from the last (most
    // keys) down, so the heaviest pairs start first, while the K/V of one chunk
    // stay in L2; or, with a.alternate, heaviest, lightest, second heaviest,
    // second lightest, ..., so that tiles finish (and their outputs leave)
    // from the start of the kernel on
    int64_t const lin = blockIdx.x / 2, per_chunk = a.head_chunk * a.q_tiles;
    int64_t const chunk = lin / per_chunk, in_chunk = lin % per_chunk;
    int64_t const chunk_bh = a.bhs - chunk * a.head_chunk < a.head_chunk ? a.bhs - chunk * a.head_chunk : a.head_chunk;
    int const order = static_cast<int>(in_chunk / chunk_bh);  // this tile's place in the dispatch order
    int const qt = a.alternate ? ((order & 1) ? order / 2 : a.q_tiles - 1 - order / 2) : a.q_tiles - 1 - order;
    int64_t const bh = chunk * a.head_chunk + in_chunk % chunk_bh;
    int64_t const hq = bh % a.Hq, b = bh / a.Hq, kvh = hq / a.g;
    int64_t const tile_q0 = static_cast<int64_t>(qt) * 2 * kBM;
    int64_t const q0 = tile_q0 + kBM * rank;  // this CTA's first query row
    int64_t const k_end = a.causal ? (a.Tk < tile_q0 + 2 * kBM ? a.Tk : tile_q0 + 2 * kBM) : a.Tk;
    int const n_kt = static_cast<int>((k_end + kBN - 1) / kBN);
    // The barriers the issuers wait on live in CTA 0; every row thread of both
    // CTAs arrives on them through the cluster window.
    uint32_t const leader_bar = map_cluster(bar, 0);
    auto signal = [&](uint32_t b_local) { mbar_arrive_cluster(leader_bar + (b_local - bar)); };

    if (tid == 0) {
        mbar_init(qready, C::ROW_ARRIVALS);
        for (int i = 0; i < 2; ++i) mbar_init(kready + 8 * i, C::ROW_ARRIVALS);
        for (int i = 0; i < 2; ++i) mbar_init(vready + 8 * i, C::ROW_ARRIVALS);
        for (int i = 0; i < 2; ++i) mbar_init(sfull + 8 * i, 1);
        for (int i = 0; i < 2; ++i) mbar_init(sfree + 8 * i, C::ROW_ARRIVALS);
        mbar_init(pfull, C::ROW_ARRIVALS);
        mbar_init(pvdone, 1);
        mbar_init(drain_s, 1);
        mbar_init(drain_pv, 1);
        for (int i = 0; i < 2; ++i) mbar_init(kfull + 8 * i, 1);
        for (int i = 0; i < 2; ++i) mbar_init(vfull + 8 * i, 1);
        fence_mbar_init();
        *abort = 0;
    }
    if (warp == 0) {
        tc::tmem_alloc_pair(smem_u32(slot), C::TMEM_COLS);
        tc::tmem_relinquish_pair();
    }
    tc::fence_before_sync();
    cluster_sync();  // both CTAs' barriers are initialised before any remote arrival
    tc::fence_after_sync();
    uint32_t const tmem = *slot;

    if (warp >= 8) {
        // ===================== MMA issue (CTA 0, warps 8 and 9) =====================
        if (lane == 0 && rank == 0) {
            // Descriptors are built once; a tile or k-step offset is added to the
            // 14-bit start-address field (shared memory is < 2^18 bytes, so the
            // field never carries).
            uint64_t const k_desc = tc::smem_desc(sbase + C::OFF_K, 16, 1024, tc::kSwizzle128B);
            uint64_t const v_desc = tc::smem_desc(sbase + C::OFF_V, C::BLK_V, 512, tc::kSwizzle128B_32B);
            uint64_t const p_desc = tc::smem_desc(sbase + C::OFF_PLO, 16, 1024, tc::kSwizzle128B);
            uint64_t const q_desc = tc::smem_desc(sbase + C::OFF_QLO, 16, 1024, tc::kSwizzle128B);
            auto at = [](uint64_t desc, uint32_t off) { return desc + static_cast<uint64_t>(off >> 4); };
            auto commit = [](uint32_t b_local) {  // this CTA's and the peer's copy of the barrier
                tc::mma_commit_pair(map_cluster(b_local, 0));
                tc::mma_commit_pair(map_cluster(b_local, 1));
            };
            auto wait = [&](uint32_t b_local, uint32_t parity) {
                return mbar_wait_or_abort<true>(b_local, parity, abort);
            };
            auto issue_s = [&](int t) {  // S = Q K^T (tile t) into S buffer t % 2
                uint32_t const kb = static_cast<uint32_t>(t & 1) * 2 * C::TILE_K;
                uint32_t const s_col = tmem + C::S_COL + kBN * static_cast<uint32_t>(t & 1);
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk) {
                    uint32_t const off = kb + (kk >> 2) * C::BLK_K + (kk & 3) * 32;
                    uint64_t const khi = at(k_desc, off), klo = at(k_desc, off + C::TILE_K);
                    uint64_t const qlo = at(q_desc, (kk >> 2) * C::QLO_BLK + (kk & 3) * 32);
                    tc::mma_tf32_ts_pair(s_col, tmem + C::Q_HI + 8 * kk, khi, C::IDESC_S, kk > 0 ? 1u : 0u);
                    tc::mma_tf32_ts_pair(s_col, tmem + C::Q_HI + 8 * kk, klo, C::IDESC_S, 1u);
                    tc::mma_tf32_ss_pair(s_col, qlo, khi, C::IDESC_S, 1u);
                }
                commit(sfull + 8 * (t & 1));
            };
            auto issue_pv = [&](int t) {  // O += P V (tile t), V from buffer t % 2
                uint32_t const vb = static_cast<uint32_t>(t & 1) * 2 * C::TILE_V;
#pragma unroll
                for (int kk = 0; kk < kBN / 8; ++kk) {
                    uint64_t const vhi = at(v_desc, vb + kk * 1024), vlo = at(v_desc, vb + C::TILE_V + kk * 1024);
                    uint64_t const plo = at(p_desc, (kk >> 2) * C::PLO_BLK + (kk & 3) * 32);
                    tc::mma_tf32_ts_pair(tmem + C::O_COL, tmem + C::P_HI + 8 * kk, vhi, C::IDESC_PV,
                                         (t > 0 || kk > 0) ? 1u : 0u);
                    tc::mma_tf32_ts_pair(tmem + C::O_COL, tmem + C::P_HI + 8 * kk, vlo, C::IDESC_PV, 1u);
                    tc::mma_tf32_ss_pair(tmem + C::O_COL, plo, vhi, C::IDESC_PV, 1u);
                }
                commit(pvdone);
            };
            if (warp == 8) {  // S(t) once K(t) is stored and softmax(t-2) has read S buffer t % 2
                bool ok = n_kt == 0 || wait(qready, 0);
                for (int t = 0; t < n_kt && ok; ++t) {
                    ok = wait(kready + 8 * (t & 1), (t >> 1) & 1) &&
                         (t < 2 || wait(sfree + 8 * (t & 1), ((t - 2) >> 1) & 1));
                    if (!ok) break;
                    tc::fence_after_sync();
                    issue_s(t);
                }
            } else {  // PV(t) once P(t) and V(t) are in place
                for (int t = 0; t < n_kt; ++t) {
                    bool const ok = wait(pfull, t & 1) && wait(vready + 8 * (t & 1), (t >> 1) & 1);
                    if (!ok) break;
                    tc::fence_after_sync();
                    issue_pv(t);
                }
            }
            // every MMA this thread issued has finished reading TMEM and shared
            // memory (of both CTAs) before either is released
            uint32_t const drain = warp == 8 ? drain_s : drain_pv;
            commit(drain);
            if (!mbar_wait_bounded(drain, 0)) *abort = 1;
        }
    } else {
        // ============================ row warps (0..7) ============================
        int const r = tid & (kBM - 1), h = tid >> 7;
        uint32_t const lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
        int64_t const qi = q0 + r;
        constexpr int HD = D / 2;  // O / Q columns per half

        // ---- K / V half tiles. K: keys [32 rank, +32) of the tile, all D dims;
        // V: all 64 keys, dims [D rank / 2, +D / 2). Element e = i * 256 + tid is
        // row e / NV4, float4 column e % NV4.
        constexpr int NV4K = D / 4, NV4V = C::VCOLS / 4;
        constexpr int PERK = C::KROWS * NV4K / kRowThreads;  // float4 per thread per tile
        constexpr int PERV = kBN * NV4V / kRowThreads;
        // Raw K and V tiles arrive by TMA (thread 0 issues). K: D / 32 boxes of 32
        // keys x 32 dims, each one 32-dim column block of the K-major 128-byte
        // swizzled layout; V: this CTA's D / 64 boxes of 64 keys x 32 dims, each
        // one column block of the MN-major layout with 32-byte atoms. The raw
        // values land where the MMA reads K_hi / V_hi, keys past Tk read as zero
        // (V rows past Tk must be finite); the row threads then add lo.
        int k_issued = 0, k_done = 0;  // K tiles issued / converted (thread 0 drains the rest)
        int v_issued = 0, v_done = 0;  // V tiles likewise
        auto issue_k = [&](int t) {    // thread 0: K(t) into buffer t % 2, once that buffer is free
            uint32_t const full_bar = kfull + 8 * (t & 1), dst = sbase + C::OFF_K + (t & 1) * 2 * C::TILE_K;
            mbar_arrive_expect_tx(full_bar, C::TILE_K);
#pragma unroll
            for (int cb = 0; cb < D / 32; ++cb)
                tma_load_4d(dst + cb * C::BLK_K, &kmap, 32 * cb, t * kBN + rank * C::KROWS, static_cast<int>(kvh),
                            static_cast<int>(b), full_bar);
            k_issued = t + 1;
        };
        auto convert_k = [&](int t) {  // K(t) has landed: lo = x - trunc13(x) beside it
            if (!mbar_wait_or_abort(kfull + 8 * (t & 1), static_cast<uint32_t>((t >> 1) & 1), abort)) return false;
            unsigned char* hi = smem + C::OFF_K + (t & 1) * 2 * C::TILE_K;
#pragma unroll
            for (int i = 0; i < PERK; ++i) {
                int const e = i * kRowThreads + tid, row = e / NV4K, c4 = e % NV4K;
                int const off = (c4 >> 3) * C::BLK_K + row * 128 + (((c4 & 7) ^ (row & 7)) << 4);
                *reinterpret_cast<float4*>(hi + C::TILE_K + off) = tf32_lo(*reinterpret_cast<float4 const*>(hi + off));
            }
            tc::fence_proxy_async_smem();  // visible to the tensor core
            k_done = t + 1;
            return true;
        };
        auto issue_v = [&](int t) {  // thread 0: V(t) into buffer t % 2, once PV(t-2) is done with it
            uint32_t const full_bar = vfull + 8 * (t & 1), dst = sbase + C::OFF_V + (t & 1) * 2 * C::TILE_V;
            mbar_arrive_expect_tx(full_bar, C::TILE_V);
#pragma unroll
            for (int cb = 0; cb < C::VCOLS / 32; ++cb)
                tma_load_4d(dst + cb * C::BLK_V, &vmap, rank * C::VCOLS + 32 * cb, t * kBN, static_cast<int>(kvh),
                            static_cast<int>(b), full_bar);
            v_issued = t + 1;
        };
        auto convert_v = [&](int t) {  // V(t) has landed: lo beside it (MN-major, 32-byte chunks XOR row % 4)
            if (!mbar_wait_or_abort(vfull + 8 * (t & 1), static_cast<uint32_t>((t >> 1) & 1), abort)) return false;
            unsigned char* hi = smem + C::OFF_V + (t & 1) * 2 * C::TILE_V;
#pragma unroll
            for (int i = 0; i < PERV; ++i) {
                int const e = i * kRowThreads + tid, row = e / NV4V, c4 = e % NV4V;
                int const off =
                    (c4 >> 3) * C::BLK_V + row * 128 + ((((c4 & 7) >> 1) ^ (row & 3)) << 5) + ((c4 & 1) << 4);
                *reinterpret_cast<float4*>(hi + C::TILE_V + off) = tf32_lo(*reinterpret_cast<float4 const*>(hi + off));
            }
            tc::fence_proxy_async_smem();
            v_done = t + 1;
            return true;
        };
        if (tid == 0) {
            for (int t = 0; t < (n_kt < 2 ? n_kt : 2); ++t) issue_k(t);
            if (n_kt > 0) issue_v(0);
        }
        {  // Q row half: hi (raw) -> TMEM, lo -> shared memory (K-major, 128-byte swizzle)
            float const* qrow = a.q + b * a.q_b + qi * a.q_t + hq * a.q_h + h * HD;
            bool const live = qi < a.Tq;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                float hi[32];
                unsigned char* qlo_row = smem + C::OFF_QLO + ((h * HD) / 32 + c) * C::QLO_BLK + r * 128;
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    float4 const x = live ? __ldg(reinterpret_cast<float4 const*>(qrow + 32 * c + j))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
                    hi[j] = x.x, hi[j + 1] = x.y, hi[j + 2] = x.z, hi[j + 3] = x.w;
                    *reinterpret_cast<float4*>(qlo_row + (((j >> 2) ^ (r & 7)) << 4)) = tf32_lo(x);
                }
                tc::tmem_st32(tmem + lane_off + C::Q_HI + h * HD + 32 * c, hi);
            }
            tc::tmem_st_wait();
            tc::fence_proxy_async_smem();
            tc::fence_before_sync();
            signal(qready);
        }
        // K runs two tiles ahead: K(0), K(1) now; K(t+2) is copied into buffer
        // t % 2 as soon as S(t) has landed and gets its lo part at the end of
        // tile t (S(t+2) is not due before S(t+1) and PV(t) have run). V runs one
        // tile ahead: V(0) now; V(t+1) is copied into buffer (t+1) % 2 once PV(t-1)
        // is done with it and gets its lo part in tile t+1 after the softmax,
        // before P(t+1) is published, so that PV(t+1) waits only for P(t+1).
        bool ok = true;
        for (int t = 0; t < (n_kt < 2 ? n_kt : 2) && ok; ++t) {
            ok = __all_sync(0xffffffffu, convert_k(t));
            if (ok) signal(kready + 8 * t);
        }
        if (ok && n_kt > 0) {
            ok = __all_sync(0xffffffffu, convert_v(0));
            if (ok) signal(vready);
        }
        unsigned char* plo_row = smem + C::OFF_PLO + h * C::PLO_BLK + r * 128;
        float const c2 = scale * kLog2e;  // scores are taken in log2 units: s * scale * log2(e)
        float m_used = Lowest<float>::value, l_part = 0.f;
        // Decisions after a wait are made warp-uniform (__all_sync): tcgen05.ld/st
        // are warp-collective, so a warp must never split on an abort.
        for (int t = 0; t < n_kt && ok; ++t) {
            uint32_t const sb = static_cast<uint32_t>(t & 1);
            ok = __all_sync(0xffffffffu, mbar_wait_or_abort(sfull + 8 * sb, (t >> 1) & 1, abort));
            if (!ok) break;  // S(t) done: K buffer t % 2 is free
            tc::fence_after_sync();
            float sv[kBN];  // [0, 32): this half's keys, [32, 64): the other half's
            uint32_t const s_col = tmem + lane_off + C::S_COL + kBN * sb;
            tc::tmem_ld32x2(s_col + 32 * h, s_col + 32 * (1 - h), sv);
            tc::fence_before_sync();
            signal(sfree + 8 * sb);  // S(t+2) may overwrite this buffer
            if (tid == 0 && t + 2 < n_kt && *abort == 0) issue_k(t + 2);  // K buffer t % 2 is free
            // live keys: kj < Tk and (not causal or kj <= qi), a prefix of the tile;
            // masking is by selects, not branches, so that the exps overlap
            int64_t const key0 = static_cast<int64_t>(t) * kBN;
            int64_t lim = a.Tk - key0;
            if (a.causal && qi + 1 - key0 < lim) lim = qi + 1 - key0;
            int const n_live = lim < 0 ? 0 : (lim > kBN ? kBN : static_cast<int>(lim));
            float part[8], pv[32];
            // interior tiles with scale >= 0 (the usual case): the max of the raw
            // scores gives the max of the scaled ones, and each exponent is one FMA
            bool const fast = c2 >= 0.f && __all_sync(0xffffffffu, n_live == kBN);
            if (fast) {
#pragma unroll
                for (int j = 0; j < kBN; ++j) part[j & 7] = j < 8 ? sv[j] : fmaxf(part[j & 7], sv[j]);
            } else {
                int const own = n_live - 32 * h, other = n_live - 32 * (1 - h);  // live counts per half
#pragma unroll
                for (int j = 0; j < kBN; ++j) {
                    sv[j] = sv[j] * c2;  // attentionScores, then ops::scale (times log2 e)
                    float const live = (j < 32 ? j < own : j - 32 < other) ? sv[j] : -INFINITY;
                    part[j & 7] = j < 8 ? live : fmaxf(part[j & 7], live);
                }
            }
            float tmax = fmaxf(fmaxf(fmaxf(part[0], part[1]), fmaxf(part[2], part[3])),
                               fmaxf(fmaxf(part[4], part[5]), fmaxf(part[6], part[7])));
            if (fast) tmax *= c2;
            // both halves see the same row and take the same decisions
            bool const grow = tmax > m_used + kLazy2;
            float alpha = 1.f;
            if (grow) {
                alpha = exp2_approx(m_used - tmax);
                m_used = tmax;
                l_part *= alpha;
            }
            if (fast) {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    pv[j] = exp2_approx(fmaf(sv[j], c2, -m_used));  // <= 2^kLazy2
                    part[j & 7] = j < 8 ? pv[j] : part[j & 7] + pv[j];
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    float const e = exp2_approx(sv[j] - m_used);
                    pv[j] = h * 32 + j < n_live ? e : 0.f;
                    part[j & 7] = j < 8 ? pv[j] : part[j & 7] + pv[j];
                }
            }
            l_part += ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
            if (t > 0) {  // V(t), copied during tile t-1: its lo part
                ok = __all_sync(0xffffffffu, convert_v(t));
                if (!ok) break;
                signal(vready + 8 * (t & 1));
            }
            // PV(t-1) has finished with V, P_hi, P_lo and O
            ok = t == 0 || mbar_wait_or_abort(pvdone, (t - 1) & 1, abort);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc::fence_after_sync();
            tc::tmem_st32(tmem + lane_off + C::P_HI + 32 * h, pv);
            // P_lo: K-major A operand, 16-byte chunk c of row r at chunk c ^ (r % 8)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                float4 const lo = tf32_lo(make_float4(pv[4 * c], pv[4 * c + 1], pv[4 * c + 2], pv[4 * c + 3]));
                *reinterpret_cast<float4*>(plo_row + ((c ^ (r & 7)) << 4)) = lo;
            }
            if (t > 0 && __any_sync(0xffffffffu, grow)) {  // this half's O columns
#pragma unroll 1
                for (int c = 0; c < HD / 32; ++c) {
                    float ov[32];
                    tc::tmem_ld32(tmem + lane_off + C::O_COL + h * HD + 32 * c, ov);
#pragma unroll
                    for (int j = 0; j < 32; ++j) ov[j] *= alpha;
                    tc::tmem_st32(tmem + lane_off + C::O_COL + h * HD + 32 * c, ov);
                }
            }
            tc::tmem_st_wait();
            tc::fence_proxy_async_smem();
            tc::fence_before_sync();
            signal(pfull);
            // V(t+1): its buffer was last read by PV(t-1), done
            if (tid == 0 && t + 1 < n_kt && *abort == 0) issue_v(t + 1);
            if (t + 2 < n_kt) {  // K(t+2), copied at the top of this tile: its lo part
                ok = __all_sync(0xffffffffu, convert_k(t + 2));
                if (!ok) break;
                signal(kready + 8 * (t & 1));
            }
        }
        if (tid == 0) {  // no K / V copy may still be landing when the CTA leaves (bounded)
            for (int t = k_done; t < k_issued; ++t)
                mbar_wait_bounded(kfull + 8 * (t & 1), static_cast<uint32_t>((t >> 1) & 1));
            for (int t = v_done; t < v_issued; ++t)
                mbar_wait_bounded(vfull + 8 * (t & 1), static_cast<uint32_t>((t >> 1) & 1));
        }
        if (ok && n_kt > 0) ok = mbar_wait_or_abort(pvdone, (n_kt - 1) & 1, abort);
        ok = __all_sync(0xffffffffu, ok);
        // row sum = the two halves' parts, exchanged through the (now idle) P_lo
        // buffer; every row thread reaches this barrier exactly once
        float* lx = reinterpret_cast<float*>(smem + C::OFF_PLO);
        if (ok) lx[tid] = l_part;
        bool const all_ok = !row_sync_any(!ok);  // the same for every row thread
        if (a.o_vec) {
            // O rows are written whole by a warp (512 contiguous bytes an
            // instruction), not 16 bytes from each of 32 rows: one packet stream to
            // the switch for a multicast output, full lines for a local one. O goes
            // through a padded staging tile over the K / V buffers, which no MMA
            // reads any more. (No system-scope fence before the CTA retires: the
            // signal barrier that follows the kernel in stream order fences, and its
            // release covers every store of this kernel. A fence in each CTA cost
            // 0.17 ms of 1.51 on the 2-GPU c3 run.)
            constexpr int PITCH = D * 4 + 16;
            unsigned char* stage = smem + C::OFF_K;
            static_assert(kBM * PITCH <= 4 * (C::TILE_K + C::TILE_V), "staging fits the K / V buffers");
            if (all_ok) {
                tc::fence_after_sync();
                float const l_sum = lx[r] + lx[r + kBM];
                float const inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
#pragma unroll 1
                for (int c = 0; c < HD / 32; ++c) {
                    int const col = h * HD + 32 * c;
                    float ov[32];
                    tc::tmem_ld32(tmem + lane_off + C::O_COL + col, ov);
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(stage + r * PITCH + (col + j) * 4) =
                            make_float4(ov[j] * inv, ov[j + 1] * inv, ov[j + 2] * inv, ov[j + 3] * inv);
                }
            }
            row_sync();
            if (all_ok) {
                constexpr int TPR = D / 4;     // threads per row, a float4 each
                constexpr int RPW = 32 / TPR;  // rows per warp instruction
                int const sub = lane / TPR, c4 = lane % TPR;
                for (int rr = warp * RPW + sub; rr < kBM; rr += 8 * RPW) {
                    int64_t const qr = q0 + rr;
                    if (qr >= a.Tq) continue;
                    float4 const val = *reinterpret_cast<float4 const*>(stage + rr * PITCH + c4 * 16);
                    int64_t const off = b * a.o_b + qr * a.o_t + hq * a.o_h + c4 * 4;
                    if (a.mirror != nullptr) mc::store(a.mirror + off, val);
                    else *reinterpret_cast<float4*>(static_cast<float*>(a.out) + off) = val;
                }
            }
        } else if (all_ok) {
            tc::fence_after_sync();
            float const l_sum = lx[r] + lx[r + kBM];
            float const inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
            int64_t const orow_off = b * a.o_b + qi * a.o_t + hq * a.o_h;
            float* orow = static_cast<float*>(a.out) + orow_off;
            float* mrow = a.mirror ? a.mirror + orow_off : nullptr;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                int const col = h * HD + 32 * c;
                float ov[32];
                tc::tmem_ld32(tmem + lane_off + C::O_COL + col, ov);
                if (qi < a.Tq) {
                    if (a.o_vec) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4*>(orow + col + j) =
                                make_float4(ov[j] * inv, ov[j + 1] * inv, ov[j + 2] * inv, ov[j + 3] * inv);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (mrow) mc::store(mrow + (col + j) * a.o_d, ov[j] * inv);
                            else orow[(col + j) * a.o_d] = ov[j] * inv;
                        }
                    }
                }
            }
        }
    }

    // CTA 1 also sees the leader's final commits land on its own barriers, so
    // that no arrival is still on its way into its shared memory when it exits.
    if (rank == 1 && warp == 8 && lane == 0)
        if (!mbar_wait_bounded(drain_s, 0) || !mbar_wait_bounded(drain_pv, 0)) *abort = 1;
    tc::fence_before_sync();
    cluster_sync();  // both CTAs are done with TMEM and shared memory of the pair
    if (*abort && tid == 0) atomicOr(&g_tc2_error, ANN_DEVERR_WAIT_TIMEOUT);
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc_pair(tmem, C::TMEM_COLS);
    }
}

template <int D>
int launch_pair(ann_stream stream, const Dims& q, const Dims& k, const Dims& v, const Dims& o, float scale,
                uint32_t g, int layout, int causal, bool& handled, void* mirror) {
    using C = PairCfg<D>;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(prefill_pair_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    if (attr != cudaSuccess) return ANN_OK;  // not handled: the single-SM kernel runs
    int const tok = layout == ANN_LAYOUT_BTHD ? 1 : 2, head = layout == ANN_LAYOUT_BTHD ? 2 : 1;
    // K [B, Tk, Hkv, D] or [B, Hkv, Tk, D] as a tensor map over (d, key, head, batch)
    int64_t const kdims[4] = {k.ext[3], k.ext[tok], k.ext[head], k.ext[0]};
    int64_t const kstr[3] = {k.str[tok], k.str[head], k.str[0]};
    if (!tma_view_ok(kdims, kstr)) return ANN_OK;  // not handled: the single-SM kernel runs
    int64_t const vdims[4] = {v.ext[3], v.ext[tok], v.ext[head], v.ext[0]};
    int64_t const vstr[3] = {v.str[tok], v.str[head], v.str[0]};
    if (!tma_view_ok(vdims, vstr)) return ANN_OK;
    CUtensorMap kmap{}, vmap{};
    ANN_TRY(map_f32_4d(&kmap, k.data, kdims, kstr, 32, C::KROWS, "attention prefill (SM pairs)"));
    ANN_TRY(map_f32_4d(&vmap, v.data, vdims, vstr, 32, kBN, "attention prefill (SM pairs)",
                       CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
    PairArgs a{};
    a.out = o.data;
    a.mirror = static_cast<float*>(mirror);
    a.q = static_cast<const float*>(q.data);
    a.k = static_cast<const float*>(k.data);
    a.v = static_cast<const float*>(v.data);
    a.q_b = q.str[0];
    a.q_t = q.str[1];
    a.q_h = q.str[2];
    a.k_b = k.str[0];
    a.k_t = k.str[tok];
    a.k_h = k.str[head];
    a.v_b = v.str[0];
    a.v_t = v.str[tok];
    a.v_h = v.str[head];
    a.o_b = o.str[0];
    a.o_t = o.str[1];
    a.o_h = o.str[2];
    a.o_d = o.str[3];
    a.o_vec = o.str[3] == 1 && reinterpret_cast<uintptr_t>(o.data) % 16 == 0 && o.str[0] % 4 == 0 &&
              o.str[1] % 4 == 0 && o.str[2] % 4 == 0 && (mirror == nullptr || aligned(mirror, 16));
    a.Tq = q.ext[1];
    a.Tk = k.ext[tok];
    a.Hq = q.ext[2];
    a.g = g;
    a.causal = causal;
    int64_t const tiles = ceil_div(a.Tq, 2 * kBM), bhs = q.ext[0] * q.ext[2];
    if (2 * tiles * bhs > INT32_MAX) return ANN_OK;  // not handled
    a.q_tiles = static_cast<int>(tiles);
    a.bhs = bhs;
    // a chunk is counted in CTAs: two per 256-row tile
    a.head_chunk = head_chunk_for(bhs, 2 * tiles, 2 * a.Tk * q.ext[3] * 4, 1);
    // ANN_PREFILL_ALTERNATE=1: query tiles alternate heavy and light. Meant for
    // a multicast output with few waves of pairs (c3 head-sharded over 8 GPUs:
    // 3.5 waves), where every tile's output must also cross NVLink into the
    // other ranks: with the heaviest tiles first nothing finishes during the
    // first wave, so the link idles and later the stores back up into the SMs.
    // A greedy-dispatch model with the link's rate puts it at 1.22 instead of
    // 1.49 x the compute time at 8 GPUs (worse at 2 GPUs); not measured on 8
    // GPUs yet, so not the default.
    if (const char* env = std::getenv("ANN_PREFILL_ALTERNATE")) a.alternate = env[0] == '1';
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute cl{};
    cl.id = cudaLaunchAttributeClusterDimension;
    cl.val.clusterDim.x = 2;
    cl.val.clusterDim.y = 1;
    cl.val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(2 * tiles * bhs));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = as_stream(stream);
    cfg.attrs = &cl;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, prefill_pair_kernel<D>, &cfg) != cudaSuccess || clusters == 0) {
        cudaGetLastError();
        return ANN_OK;  // not handled
    }
    handled = true;
    cudaError_t const e = cudaLaunchKernelEx(&cfg, prefill_pair_kernel<D>, a, scale, kmap, vmap);
    if (e != cudaSuccess) return fail(ANN_ECUDA, "attention prefill (SM pairs): %s", cudaGetErrorString(e));
    return check_launch("attention prefill (SM pairs)");
}

}  // namespace

// fp32 prefill on pairs of SMs for D 64 / 128 (the caller has checked unit-stride,
// 16-byte aligned Q/K/V rows); `handled` = false when it does not run (other D,
// ANN_PREFILL_TC_PAIR=0, or no 2-CTA cluster of it can be resident).
int prefill_tc_pair_f32(ann_stream stream, const Dims& q, const Dims& k, const Dims& v, const Dims& o, float scale,
                        uint32_t g, int layout, int causal, bool& handled, void* mirror) {
    handled = false;
    if (const char* env = std::getenv("ANN_PREFILL_TC_PAIR"))
        if (env[0] == '0' && mirror == nullptr) return ANN_OK;
    if (q.ext[3] == 64) return launch_pair<64>(stream, q, k, v, o, scale, g, layout, causal, handled, mirror);
    if (q.ext[3] == 128) return launch_pair<128>(stream, q, k, v, o, scale, g, layout, causal, handled, mirror);
    return ANN_OK;
}

int take_prefill_tc2_error(cudaStream_t s, uint32_t* bits) {
    unsigned int value = 0, zero = 0;
    if (cudaMemcpyFromSymbolAsync(&value, g_tc2_error, sizeof value, 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_tc2_error, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ANN_ECUDA, "device error word: %s", cudaGetErrorString(cudaGetLastError()));
    *bits |= value;
    return ANN_OK;
}

}  // namespace ann
