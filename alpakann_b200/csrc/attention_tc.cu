// attention_tc.cu -- the drop-in attentionScores / attentionApply (fp32) on the
// tensor cores: tcgen05 kind::tf32 with the 3xTF32 split, on pairs of SMs.
//
// Reference: onHost/nn/attention.hpp:54-110, onAcc/internal/nn/attention.hpp:15-68
// (composed per op in test/unit/nn/attention.cpp:591-651). Both ops are batched
// contractions per (batch, query head), KV head hq / queriesPerKvGroup:
//   scores: S[b,hq,i,j] = sum_d Q[b,i,hq,d] K[b,j,kvh,d]   (unscaled)
//   apply:  O[b,i,hq,d] = sum_j P[b,hq,i,j] V[b,j,kvh,d]
// 3xTF32 as in the fused prefill (prefill_tc2.cu): x = hi + lo, hi = the raw
// fp32 value (the MMA reads its top 19 bits), lo = x - trunc13(x), exact;
// A.B = A_hi B_hi + A_hi B_lo + A_lo B_hi with fp32 accumulation in TMEM.
//
// A cluster of two CTAs owns 256 rows (CTA r: rows [128 r, 128 r + 128)); one
// thread of CTA 0 issues M = 256 MMAs (cta_group::2) for both, each CTA holds
// half of every B tile. Row threads (warps 0..7 of both CTAs) stage operands
// and signal CTA 0's barriers through the cluster window; the issuer commits
// each MMA group to both CTAs' barriers. Every wait is bounded: on a timeout
// the CTAs stop, the issuer drains its MMAs, both meet at a cluster barrier,
// free TMEM and report ANN_DEVERR_WAIT_TIMEOUT.
//
// scores_pair_kernel: Q (hi and lo) in TMEM as the A operand for the CTA's
//   whole life; 128-key K tiles (each CTA 64 keys, raw by TMA tensor loads +
//   lo added by the row threads, K-major 128-byte swizzle) two buffers deep; S accumulators double-buffered in TMEM. The
//   epilogue moves S rows TMEM -> registers -> two 32-row x 32-key staging
//   boxes per warp (128-byte swizzle) -> one TMA tensor store per box, issued
//   by the warp itself, which clips rows past Tq and keys past Tk. Work unit:
//   (batch*head, 256-row tile, key chunk).
// apply_pair_kernel: a copy warp brings 64-key chunks of P into a 4-deep
//   ring of shared-memory stages (one bulk copy per 256-byte row piece, rows
//   padded by 16 bytes), so P, the large operand, is always several chunks in
//   flight without passing through registers; each row thread reads its row
//   back, splits it into hi / lo and stores both into TMEM (the A operand); V
//   chunks (each CTA half of the head dims, raw + lo, MN-major 32-byte-atom
//   swizzle) two buffers deep; O accumulates in TMEM.
//   With few tiles the key range is split in two and both halves add into a
//   zeroed output (red.global.add: 0 + a + b in either order is a + b, so the
//   result does not depend on which half finishes first).
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"
#include "tmap.cuh"

namespace ann {

int scores_tc_f32(ann_stream stream, const Dims& q, const Dims& k, const Dims& s, uint32_t g, int layout,
                  bool& handled);
int apply_tc_f32(ann_stream stream, const Dims& p, const Dims& v, const Dims& o, uint32_t g, int layout,
                 bool& handled);
int take_attention_tc_error(cudaStream_t s, uint32_t* bits);

namespace {

__device__ unsigned int g_atc_error;

constexpr int kBM = 128;                    // rows per CTA
constexpr int kRowThreads = 256;            // warps 0..7
constexpr int kThreads = kRowThreads + 32;  // + warp 8 (MMA issuer)

__device__ __forceinline__ float tf32_lo(float x) {
    return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}
__device__ __forceinline__ float4 tf32_lo(float4 x) {
    return make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
}
// A barrier of the 256 row threads of this CTA that also ORs `v` over them:
// every one gets the same answer
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
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ============================================================================
// attentionScores
// ============================================================================
template <int D>
struct ScCfg {
    static constexpr int NT = 128;                  // keys per tile (MMA N)
    static constexpr int KROWS = NT / 2;            // keys of a tile held by this CTA
    static constexpr int TILE_K = KROWS * D * 4;    // bytes of K hi (or lo) per buffer
    static constexpr int BLK_K = KROWS * 128;       // one 32-float column block of K
    static constexpr int BOX_S = 32 * 128;          // one TMA box of S: 32 rows x 32 keys, 128-byte swizzle
    static constexpr int OFF_K = 0;                 // buffer i: hi at 2*i*TILE_K, lo at + TILE_K
    static constexpr int OFF_ST = 4 * TILE_K;       // S staging: two boxes per row warp
    static constexpr int OFF_BAR = OFF_ST + 16 * BOX_S;
    // barriers: qready kready[2] sfree[2] sfull[2] drain kfull[2]
    static constexpr int NBAR = 10;
    static constexpr int OFF_SLOT = OFF_BAR + NBAR * 8;  // TMEM base, abort flag
    static constexpr int USED = OFF_SLOT + 16;
    static constexpr int SMEM = USED + 1024;  // + 1 KB to align the base to the swizzle atom
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static constexpr uint32_t Q_HI = 0, Q_LO = D, S_COL = 2 * D;  // S buffer b at S_COL + NT b
    static constexpr uint32_t TMEM_COLS = 512;
    static_assert(S_COL + 2 * NT <= TMEM_COLS, "TMEM budget");
    static constexpr uint32_t IDESC = tc::idesc_tf32(2 * kBM, NT, false);
    static constexpr uint32_t ROW_ARRIVALS = 2 * kRowThreads;
};

struct ScArgs {
    const float* q;
    const float* k;
    float* s;
    int64_t q_b, q_t, q_h;  // element strides (unit along d)
    int64_t k_b, k_t, k_h;
    int64_t s_b, s_h, s_t;  // unit along keys
    int64_t Tq, Tk, Hq;
    uint32_t g;
    int q_tiles;   // 256-row tiles
    int k_tiles;   // 128-key tiles in all
    int chunk;     // key tiles per work unit
    int chunks;    // work units along the keys
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1) scores_pair_kernel(ScArgs a, const __grid_constant__ CUtensorMap smap,
                                                                  const __grid_constant__ CUtensorMap kmap) {
    using C = ScCfg<D>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    uint32_t const raw_base = smem_u32(smem_raw);
    uint32_t const pad = (1024u - (raw_base & 1023u)) & 1023u;
    unsigned char* smem = smem_raw + pad;
    uint32_t const sbase = raw_base + pad;
    uint32_t const bar = sbase + C::OFF_BAR;
    uint32_t const qready = bar, kready = bar + 8, sfree = bar + 24, sfull = bar + 40, drain = bar + 56,
                   kfull = bar + 64;
    uint32_t* slot = reinterpret_cast<uint32_t*>(smem + C::OFF_SLOT);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + C::OFF_SLOT + 4);

    int const tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int const rank = static_cast<int>(cluster_ctarank());
    // work unit: key chunk fastest, then the 256-row tile, then (batch, head)
    int64_t const unit = blockIdx.x / 2;
    int const kc = static_cast<int>(unit % a.chunks);
    int64_t const rest = unit / a.chunks;
    int const qt = static_cast<int>(rest % a.q_tiles);
    int64_t const bh = rest / a.q_tiles;
    int64_t const hq = bh % a.Hq, b = bh / a.Hq, kvh = hq / a.g;
    int64_t const q0 = static_cast<int64_t>(qt) * 2 * kBM + kBM * rank;  // this CTA's first row
    int const t_begin = kc * a.chunk;
    int const n_t = (a.k_tiles - t_begin < a.chunk ? a.k_tiles - t_begin : a.chunk);
    uint32_t const leader_bar = map_cluster(bar, 0);
    auto signal = [&](uint32_t b_local) { mbar_arrive_cluster(leader_bar + (b_local - bar)); };

    if (tid == 0) {
        mbar_init(qready, C::ROW_ARRIVALS);
        for (int i = 0; i < 2; ++i) mbar_init(kready + 8 * i, C::ROW_ARRIVALS);
        for (int i = 0; i < 2; ++i) mbar_init(sfree + 8 * i, C::ROW_ARRIVALS);
        for (int i = 0; i < 2; ++i) mbar_init(sfull + 8 * i, 1);
        mbar_init(drain, 1);
        for (int i = 0; i < 2; ++i) mbar_init(kfull + 8 * i, 1);
        fence_mbar_init();
        *abort = 0;
    }
    if (warp == 0) {
        tc::tmem_alloc_pair(smem_u32(slot), C::TMEM_COLS);
        tc::tmem_relinquish_pair();
    }
    tc::fence_before_sync();
    cluster_sync();
    tc::fence_after_sync();
    uint32_t const tmem = *slot;

    if (warp == 8) {
        // ============================ MMA issue (CTA 0) ============================
        // One issuer: S(t) and S(t+1) complete in order. (A second issuer taking
        // the odd tiles let their MMAs interleave in the tensor pipe, so both
        // buffers finished late and the epilogue could not overlap: measured
        // slower, 154 against 166 TFLOP/s at [1,8,4096,4096] x 128.)
        if (lane == 0 && rank == 0) {
            uint64_t const k_desc = tc::smem_desc(sbase + C::OFF_K, 16, 1024, tc::kSwizzle128B);
            auto at = [](uint64_t desc, uint32_t off) { return desc + static_cast<uint64_t>(off >> 4); };
            auto commit = [](uint32_t b_local) {
                tc::mma_commit_pair(map_cluster(b_local, 0));
                tc::mma_commit_pair(map_cluster(b_local, 1));
            };
            auto wait = [&](uint32_t b_local, uint32_t parity) {
                return mbar_wait_or_abort<true>(b_local, parity, abort);
            };
            bool ok = n_t <= 0 || wait(qready, 0);
            for (int t = 0; t < n_t && ok; ++t) {
                ok = wait(kready + 8 * (t & 1), (t >> 1) & 1) && (t < 2 || wait(sfree + 8 * (t & 1), ((t - 2) >> 1) & 1));
                if (!ok) break;
                tc::fence_after_sync();
                uint32_t const kb = static_cast<uint32_t>(t & 1) * 2 * C::TILE_K;
                uint32_t const s_col = tmem + C::S_COL + C::NT * static_cast<uint32_t>(t & 1);
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk) {
                    uint32_t const off = kb + (kk >> 2) * C::BLK_K + (kk & 3) * 32;
                    uint64_t const khi = at(k_desc, off), klo = at(k_desc, off + C::TILE_K);
                    tc::mma_tf32_ts_pair(s_col, tmem + C::Q_HI + 8 * kk, khi, C::IDESC, kk > 0 ? 1u : 0u);
                    tc::mma_tf32_ts_pair(s_col, tmem + C::Q_HI + 8 * kk, klo, C::IDESC, 1u);
                    tc::mma_tf32_ts_pair(s_col, tmem + C::Q_LO + 8 * kk, khi, C::IDESC, 1u);
                }
                commit(sfull + 8 * (t & 1));
            }
            commit(drain);
            if (!mbar_wait_bounded(drain, 0)) *abort = 1;
        }
    } else {
        // ============================ row warps (0..7) ============================
        int const r = tid & (kBM - 1), h = tid >> 7;
        uint32_t const lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
        int64_t const qi = q0 + r;
        constexpr int NV4 = D / 4;                                // float4 per K row
        constexpr int PERK = C::KROWS * NV4 / kRowThreads;        // float4 per thread per tile
        // Raw K tiles (keys [NT t + KROWS rank, + KROWS) of tile t) arrive by TMA,
        // D / 32 boxes of KROWS keys x 32 dims, each one column block of the
        // K-major 128-byte-swizzled K_hi layout (keys past Tk read as zero);
        // the row threads add lo beside them.
        int k_issued = 0, k_done = 0;  // K tiles issued / converted (thread 0 drains the rest)
        auto issue_k = [&](int t) {    // thread 0: K(t) into buffer t % 2, once S(t-2) has read it
            uint32_t const full_bar = kfull + 8 * (t & 1), dst = sbase + C::OFF_K + (t & 1) * 2 * C::TILE_K;
            mbar_arrive_expect_tx(full_bar, C::TILE_K);
#pragma unroll
            for (int cb = 0; cb < D / 32; ++cb)
                tma_load_4d(dst + cb * C::BLK_K, &kmap, 32 * cb, (t_begin + t) * C::NT + rank * C::KROWS,
                            static_cast<int>(kvh), static_cast<int>(b), full_bar);
            k_issued = t + 1;
        };
        auto convert_k = [&](int t) {  // K(t) has landed: lo = x - trunc13(x) beside it
            if (!mbar_wait_or_abort(kfull + 8 * (t & 1), static_cast<uint32_t>((t >> 1) & 1), abort)) return false;
            unsigned char* hi = smem + C::OFF_K + (t & 1) * 2 * C::TILE_K;
#pragma unroll
            for (int i = 0; i < PERK; ++i) {
                int const e = i * kRowThreads + tid, row = e / NV4, c4 = e % NV4;
                int const off = (c4 >> 3) * C::BLK_K + row * 128 + (((c4 & 7) ^ (row & 7)) << 4);
                *reinterpret_cast<float4*>(hi + C::TILE_K + off) = tf32_lo(*reinterpret_cast<float4 const*>(hi + off));
            }
            tc::fence_proxy_async_smem();
            k_done = t + 1;
            return true;
        };
        if (tid == 0)
            for (int t = 0; t < (n_t < 2 ? n_t : 2); ++t) issue_k(t);
        {  // Q row half -> TMEM: hi (raw) at Q_HI, lo at Q_LO
            constexpr int HD = D / 2;
            float const* qrow = a.q + b * a.q_b + qi * a.q_t + hq * a.q_h + h * HD;
            bool const live = qi < a.Tq;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                float hi[32], lo[32];
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    float4 const x = live ? __ldg(reinterpret_cast<float4 const*>(qrow + 32 * c + j))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
                    float4 const y = tf32_lo(x);
                    hi[j] = x.x, hi[j + 1] = x.y, hi[j + 2] = x.z, hi[j + 3] = x.w;
                    lo[j] = y.x, lo[j + 1] = y.y, lo[j + 2] = y.z, lo[j + 3] = y.w;
                }
                tc::tmem_st32(tmem + lane_off + C::Q_HI + h * HD + 32 * c, hi);
                tc::tmem_st32(tmem + lane_off + C::Q_LO + h * HD + 32 * c, lo);
            }
            tc::tmem_st_wait();
            tc::fence_before_sync();
            signal(qready);
        }
        bool ok = true;
        for (int t = 0; t < (n_t < 2 ? n_t : 2) && ok; ++t) {
            ok = __all_sync(0xffffffffu, convert_k(t));
            if (ok) signal(kready + 8 * t);
        }
        // S leaves through two staging boxes per warp (its 32 rows x the 64
        // keys of this half: 32 keys a box) and one TMA store per box, issued
        // by the warp's lane 0 once the warp has staged them; the store clips
        // rows past Tq and keys past Tk.
        unsigned char* st_row = smem + C::OFF_ST + 2 * warp * C::BOX_S + lane * 128;
        uint32_t const st_warp = sbase + C::OFF_ST + 2 * warp * C::BOX_S;
        int64_t const row0 = q0 + 32 * (warp & 3);  // the warp's first row
        for (int t = 0; t < n_t && ok; ++t) {
            uint32_t const sb = static_cast<uint32_t>(t & 1);
            ok = __all_sync(0xffffffffu, mbar_wait_or_abort(sfull + 8 * sb, (t >> 1) & 1, abort));
            if (!ok) break;  // warp-uniform: the TMEM loads below are warp-collective
            tc::fence_after_sync();  // S(t) done: K buffer t % 2 is free
            if (tid == 0 && t + 2 < n_t && *abort == 0) issue_k(t + 2);
            float sv[64];  // this thread's half of row r: keys [64 h, 64 h + 64) of the tile
            uint32_t const s_col = tmem + lane_off + C::S_COL + C::NT * sb + 64 * h;
            tc::tmem_ld32x2(s_col, s_col + 32, sv);
            tc::fence_before_sync();
            signal(sfree + 8 * sb);
            if (lane == 0) bulk_wait_read();  // the warp's previous stores have read its boxes
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 16; ++j)  // piece j of the 64 keys: box j / 8, piece j % 8
                *reinterpret_cast<float4*>(st_row + (j >> 3) * C::BOX_S + (((j & 7) ^ (lane & 7)) << 4)) =
                    make_float4(sv[4 * j], sv[4 * j + 1], sv[4 * j + 2], sv[4 * j + 3]);
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                int64_t const key0 = static_cast<int64_t>(t_begin + t) * C::NT + 64 * h;
#pragma unroll
                for (int x = 0; x < 2; ++x)
                    if (key0 + 32 * x < a.Tk && row0 < a.Tq)  // boxes wholly outside are not issued
                        tma_store_4d(&smap, static_cast<int>(key0 + 32 * x), static_cast<int>(row0),
                                     static_cast<int>(hq), static_cast<int>(b), st_warp + x * C::BOX_S);
                bulk_commit();
            }
            if (t + 2 < n_t) {  // K(t+2), copied at the top of this tile: its lo part
                ok = __all_sync(0xffffffffu, convert_k(t + 2));
                if (!ok) break;
                signal(kready + 8 * (t & 1));
            }
        }
        if (lane == 0) bulk_wait_all();
        if (tid == 0)  // no K copy may still be landing when the CTA leaves (bounded)
            for (int t = k_done; t < k_issued; ++t)
                mbar_wait_bounded(kfull + 8 * (t & 1), static_cast<uint32_t>((t >> 1) & 1));
    }

    // CTA 1 also sees the issuer's final commit land on its own barrier, so that
    // no arrival is still on its way into its shared memory when it exits
    if (rank == 1 && warp == 8 && lane == 0 && !mbar_wait_bounded(drain, 0)) *abort = 1;
    tc::fence_before_sync();
    cluster_sync();  // both CTAs are done with TMEM and shared memory of the pair
    if (*abort && tid == 0) atomicOr(&g_atc_error, ANN_DEVERR_WAIT_TIMEOUT);
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc_pair(tmem, C::TMEM_COLS);
    }
}

// ============================================================================
// attentionApply
// ============================================================================
template <int D>
struct ApCfg {
    static constexpr int KC = 64;                  // keys per chunk (MMA K = 8 x 8)
    static constexpr int VCOLS = D / 2;            // head dims of a V chunk held by this CTA
    static constexpr int TILE_V = KC * VCOLS * 4;  // bytes of V hi (or lo) per buffer
    static constexpr int BLK_V = KC * 128;         // one 32-float column block of V
    static constexpr int BOX_P = kBM * 128;        // one TMA box of P: 128 rows x 32 keys, 128-byte swizzle
    static constexpr int STAGE_P = 2 * BOX_P;      // one P chunk: keys [0, 32) and [32, 64)
    static constexpr int NST = 4;                  // P stages
    static constexpr int OFF_V = 0;                // buffer i: hi at 2*i*TILE_V, lo at + TILE_V
    static constexpr int OFF_P = 4 * TILE_V;       // stage i at OFF_P + i*STAGE_P
    static constexpr int OFF_BAR = OFF_P + NST * STAGE_P;
    // barriers: pready[2] pvdone[2] drain pfull[NST] pfree[NST]
    static constexpr int NBAR = 5 + 2 * NST;
    static constexpr int OFF_SLOT = OFF_BAR + NBAR * 8;
    static constexpr int USED = OFF_SLOT + 16;
    // >= 120 KB: one CTA per SM, so that its TMEM allocation never waits
    static constexpr int SMEM = USED + 1024 > 120 * 1024 ? USED + 1024 : 120 * 1024;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static constexpr uint32_t O_COL = 0, P_HI = D, P_LO = D + 2 * KC;  // buffer b at + KC b
    static constexpr uint32_t TMEM_COLS = 512;
    static_assert(P_LO + 2 * KC <= TMEM_COLS, "TMEM budget");
    static constexpr uint32_t IDESC = tc::idesc_tf32(2 * kBM, D, true);
    static constexpr uint32_t ROW_ARRIVALS = 2 * kRowThreads;
};
constexpr int kApThreads = kRowThreads + 64;  // + warp 8 (MMA issuer) and warp 9 (P copies)

struct ApArgs {
    const float* p;
    const float* v;
    float* o;
    int64_t p_b, p_h, p_t;  // unit along keys
    int64_t v_b, v_t, v_h;  // unit along d
    int64_t o_b, o_t, o_h;  // unit along d
    int64_t Tq, Tk, Hq;
    uint32_t g;
    int q_tiles;
    int splits;  // 1, or 2 halves of the key range adding into a zeroed output
    int64_t chunks;  // KC-key chunks in all
};

template <int D>
__global__ void __launch_bounds__(kApThreads, 1) apply_pair_kernel(ApArgs a, const __grid_constant__ CUtensorMap pmap) {
    using C = ApCfg<D>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    uint32_t const raw_base = smem_u32(smem_raw);
    uint32_t const pad = (1024u - (raw_base & 1023u)) & 1023u;
    unsigned char* smem = smem_raw + pad;
    uint32_t const sbase = raw_base + pad;
    uint32_t const bar = sbase + C::OFF_BAR;
    uint32_t const pready = bar, pvdone = bar + 16, drain = bar + 32, pfull = bar + 40, pfree = pfull + 8 * C::NST;
    uint32_t* slot = reinterpret_cast<uint32_t*>(smem + C::OFF_SLOT);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + C::OFF_SLOT + 4);

    int const tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int const rank = static_cast<int>(cluster_ctarank());
    int64_t const unit = blockIdx.x / 2;
    int const split = static_cast<int>(unit % a.splits);
    int64_t const rest = unit / a.splits;
    int const qt = static_cast<int>(rest % a.q_tiles);
    int64_t const bh = rest / a.q_tiles;
    int64_t const hq = bh % a.Hq, b = bh / a.Hq, kvh = hq / a.g;
    int64_t const q0 = static_cast<int64_t>(qt) * 2 * kBM + kBM * rank;
    int64_t const per = (a.chunks + a.splits - 1) / a.splits;
    int64_t const c_begin = split * per;
    int const n_c = static_cast<int>(a.chunks - c_begin < per ? a.chunks - c_begin : per);
    uint32_t const leader_bar = map_cluster(bar, 0);
    auto signal = [&](uint32_t b_local) { mbar_arrive_cluster(leader_bar + (b_local - bar)); };

    if (tid == 0) {
        for (int i = 0; i < 2; ++i) mbar_init(pready + 8 * i, C::ROW_ARRIVALS);
        for (int i = 0; i < 2; ++i) mbar_init(pvdone + 8 * i, 1);
        mbar_init(drain, 1);
        for (int i = 0; i < C::NST; ++i) mbar_init(pfull + 8 * i, 1);
        for (int i = 0; i < C::NST; ++i) mbar_init(pfree + 8 * i, kRowThreads);
        fence_mbar_init();
        *abort = 0;
    }
    if (warp == 0) {
        tc::tmem_alloc_pair(smem_u32(slot), C::TMEM_COLS);
        tc::tmem_relinquish_pair();
    }
    tc::fence_before_sync();
    cluster_sync();
    tc::fence_after_sync();
    uint32_t const tmem = *slot;

    if (warp == 8) {
        if (lane == 0 && rank == 0) {
            uint64_t const v_desc = tc::smem_desc(sbase + C::OFF_V, C::BLK_V, 512, tc::kSwizzle128B_32B);
            auto at = [](uint64_t desc, uint32_t off) { return desc + static_cast<uint64_t>(off >> 4); };
            auto commit = [](uint32_t b_local) {
                tc::mma_commit_pair(map_cluster(b_local, 0));
                tc::mma_commit_pair(map_cluster(b_local, 1));
            };
            for (int c = 0; c < n_c; ++c) {
                if (!mbar_wait_or_abort<true>(pready + 8 * (c & 1), (c >> 1) & 1, abort)) break;
                tc::fence_after_sync();
                uint32_t const vb = static_cast<uint32_t>(c & 1) * 2 * C::TILE_V;
                uint32_t const pcol = C::KC * static_cast<uint32_t>(c & 1);
#pragma unroll
                for (int kk = 0; kk < C::KC / 8; ++kk) {
                    uint64_t const vhi = at(v_desc, vb + kk * 1024), vlo = at(v_desc, vb + C::TILE_V + kk * 1024);
                    uint32_t const phi = tmem + C::P_HI + pcol + 8 * kk, plo = tmem + C::P_LO + pcol + 8 * kk;
                    tc::mma_tf32_ts_pair(tmem + C::O_COL, phi, vhi, C::IDESC, (c > 0 || kk > 0) ? 1u : 0u);
                    tc::mma_tf32_ts_pair(tmem + C::O_COL, phi, vlo, C::IDESC, 1u);
                    tc::mma_tf32_ts_pair(tmem + C::O_COL, plo, vhi, C::IDESC, 1u);
                }
                commit(pvdone + 8 * (c & 1));
            }
            commit(drain);
            if (!mbar_wait_bounded(drain, 0)) *abort = 1;
        }
    } else if (warp == 9) {
        // P of this CTA's 128 query rows, chunk by chunk, into an NST-deep ring
        // of stages: two TMA boxes a chunk (128 rows x 32 keys each, 128-byte
        // swizzle: 16-byte piece j of row r at r * 128 + ((j ^ (r % 8)) << 4)).
        // Rows past Tq and keys past Tk arrive as zeros.
        if (lane == 0) {
            int issued = 0;
            for (int c = 0; c < n_c; ++c) {
                int const st = c % C::NST;
                if (c >= C::NST && !mbar_wait_or_abort(pfree + 8 * st, ((c - C::NST) / C::NST) & 1, abort)) break;
                int const key0 = static_cast<int>((c_begin + c) * C::KC);
                uint32_t const full_bar = pfull + 8 * st, dst = sbase + C::OFF_P + st * C::STAGE_P;
                mbar_arrive_expect_tx(full_bar, C::STAGE_P);
                tma_load_4d(dst, &pmap, key0, static_cast<int>(q0), static_cast<int>(hq), static_cast<int>(b),
                            full_bar);
                tma_load_4d(dst + C::BOX_P, &pmap, key0 + 32, static_cast<int>(q0), static_cast<int>(hq),
                            static_cast<int>(b), full_bar);
                issued = c + 1;
            }
            // every copy has landed before the CTA can exit (the row threads
            // have waited for all of them, unless they stopped early); bounded
            for (int c = issued - C::NST < 0 ? 0 : issued - C::NST; c < issued; ++c)
                mbar_wait_bounded(pfull + 8 * (c % C::NST), static_cast<uint32_t>((c / C::NST) & 1));
        }
    } else {
        int const r = tid & (kBM - 1), h = tid >> 7;
        uint32_t const lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
        int64_t const qi = q0 + r;
        constexpr int NV4V = C::VCOLS / 4;
        constexpr int PERV = C::KC * NV4V / kRowThreads;  // 2 (D 64) or 4 (D 128)
        static_assert(PERV >= 1, "V chunk per thread");
        float const* vbase = a.v + b * a.v_b + kvh * a.v_h + rank * C::VCOLS;
        float4 rv[PERV];
        auto load_v = [&](int c) {
            int64_t const key0 = (c_begin + c) * C::KC;
#pragma unroll
            for (int i = 0; i < PERV; ++i) {
                int const e = i * kRowThreads + tid, row = e / NV4V, c4 = e % NV4V;
                int64_t const key = key0 + row;
                rv[i] = key < a.Tk ? __ldg(reinterpret_cast<float4 const*>(vbase + key * a.v_t) + c4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);  // V rows past Tk must be finite
            }
        };
        auto stage_v = [&](int buf) {  // V hi / lo (MN-major, 32-byte chunks XOR row % 4)
            unsigned char* hi = smem + C::OFF_V + buf * 2 * C::TILE_V;
#pragma unroll
            for (int i = 0; i < PERV; ++i) {
                int const e = i * kRowThreads + tid, row = e / NV4V, c4 = e % NV4V;
                int const off =
                    (c4 >> 3) * C::BLK_V + row * 128 + ((((c4 & 7) >> 1) ^ (row & 3)) << 5) + ((c4 & 1) << 4);
                *reinterpret_cast<float4*>(hi + off) = rv[i];
                *reinterpret_cast<float4*>(hi + C::TILE_V + off) = tf32_lo(rv[i]);
            }
            tc::fence_proxy_async_smem();
        };
        if (n_c > 0) load_v(0);
        bool ok = true;
        for (int c = 0; c < n_c; ++c) {
            int const buf = c & 1, st = c % C::NST;
            // TMEM P buffer and V buffer `buf` were last read by PV(c-2); P chunk c
            // has landed. The decision to stop is taken by all row threads
            // together, since they meet at the barriers below.
            bool fail = c >= 2 && !mbar_wait_or_abort(pvdone + 8 * buf, ((c - 2) >> 1) & 1, abort);
            if (!fail) fail = !mbar_wait_or_abort(pfull + 8 * st, static_cast<uint32_t>((c / C::NST) & 1), abort);
            if (row_sync_any(fail || *abort != 0)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            stage_v(buf);
            if (c + 1 < n_c) load_v(c + 1);
            {  // this thread's 32 keys of row r (box h): hi -> TMEM P_HI, lo -> TMEM P_LO
                unsigned char const* prow = smem + C::OFF_P + st * C::STAGE_P + h * C::BOX_P + r * 128;
                float hi[32], lo[32];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float4 const x = *reinterpret_cast<float4 const*>(prow + ((j ^ (r & 7)) << 4));
                    float4 const y = tf32_lo(x);
                    hi[4 * j] = x.x, hi[4 * j + 1] = x.y, hi[4 * j + 2] = x.z, hi[4 * j + 3] = x.w;
                    lo[4 * j] = y.x, lo[4 * j + 1] = y.y, lo[4 * j + 2] = y.z, lo[4 * j + 3] = y.w;
                }
                mbar_arrive(pfree + 8 * st);  // the stage may take chunk c + NST
                uint32_t const col = C::KC * static_cast<uint32_t>(buf) + 32 * h;
                tc::tmem_st32(tmem + lane_off + C::P_HI + col, hi);
                tc::tmem_st32(tmem + lane_off + C::P_LO + col, lo);
            }
            tc::tmem_st_wait();
            tc::fence_before_sync();
            signal(pready + 8 * buf);
        }
        if (ok && n_c > 0) ok = mbar_wait_or_abort(pvdone + 8 * ((n_c - 1) & 1), ((n_c - 1) >> 1) & 1, abort);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {  // warp-uniform: the TMEM loads are warp-collective, only the stores are per row
            tc::fence_after_sync();
            constexpr int HD = D / 2;
            float* orow = a.o + b * a.o_b + qi * a.o_t + hq * a.o_h + h * HD;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                float ov[32];
                tc::tmem_ld32(tmem + lane_off + C::O_COL + h * HD + 32 * c, ov);
                if (qi < a.Tq) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float* dst = orow + 32 * c + j;
                        if (a.splits == 1) {
                            *reinterpret_cast<float4*>(dst) = make_float4(ov[j], ov[j + 1], ov[j + 2], ov[j + 3]);
                        } else {
                            asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(ov[j]),
                                         "f"(ov[j + 1]), "f"(ov[j + 2]), "f"(ov[j + 3])
                                         : "memory");
                        }
                    }
                }
            }
        }
    }

    if (rank == 1 && warp == 8 && lane == 0 && !mbar_wait_bounded(drain, 0)) *abort = 1;
    tc::fence_before_sync();
    cluster_sync();
    if (*abort && tid == 0) atomicOr(&g_atc_error, ANN_DEVERR_WAIT_TIMEOUT);
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc_pair(tmem, C::TMEM_COLS);
    }
}

template <typename K, typename... A>
int cluster_launch(K kernel, int threads, int smem, int64_t ctas, ann_stream stream, const char* what,
                   A const&... args) {
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute cl{};
    cl.id = cudaLaunchAttributeClusterDimension;
    cl.val.clusterDim.x = 2;
    cl.val.clusterDim.y = 1;
    cl.val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(ctas));
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = as_stream(stream);
    cfg.attrs = &cl;
    cfg.numAttrs = 1;
    cudaError_t const e = cudaLaunchKernelEx(&cfg, kernel, args...);
    if (e != cudaSuccess) return fail(ANN_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return check_launch(what);
}

bool tc_disabled() {
    const char* env = std::getenv("ANN_ATTENTION_OPS_SIMT");
    return env != nullptr && env[0] == '1';
}

// Tensor map of an fp32 [B, H, T, K] view (K innermost) with the given
// extents, boxes of box_rows rows x 32 keys (tmap.cuh).
int map_bhtk(const float* base, int64_t B, int64_t H, int64_t T, int64_t K, int64_t s_b, int64_t s_h, int64_t s_t,
             uint32_t box_rows, CUtensorMap* map, const char* what) {
    return map_f32_4d(map, base, {K, T, H, B}, {s_t, s_h, s_b}, 32, box_rows, what);
}

bool tma_view(const Dims& d) {  // a [B, H, T, K] view with unit-stride K
    return tma_view_ok({d.ext[3], d.ext[2], d.ext[1], d.ext[0]}, {d.str[2], d.str[1], d.str[0]});
}

template <int D>
int launch_scores(ann_stream stream, ScArgs& a, int64_t bhs, int64_t const (&kdims)[4], int64_t const (&kstr)[3]) {
    using C = ScCfg<D>;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(scores_pair_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    if (attr != cudaSuccess) return fail(ANN_ECUDA, "attentionScores (tensor cores) setup: %s", cudaGetErrorString(attr));
    // key tiles per work unit: the smallest chunk from 4 to 16 tiles whose
    // grid has no short last wave of pairs (a chunk's fixed cost is loading Q)
    int64_t const slots = sm_count() / 2;
    int best = a.k_tiles < 16 ? a.k_tiles : 16;
    double best_cost = 1e300;
    for (int ch = 4; ch <= 16; ++ch) {
        int const c = ch < a.k_tiles ? ch : a.k_tiles;
        int64_t const units = bhs * a.q_tiles * ceil_div(a.k_tiles, c);
        double const cost = static_cast<double>(ceil_div(units, slots)) * (c + 1.5);
        if (cost < best_cost - 1e-9) best_cost = cost, best = c;
        if (c == a.k_tiles) break;
    }
    a.chunk = best;
    a.chunks = static_cast<int>(ceil_div(a.k_tiles, best));
    int64_t const ctas = 2 * bhs * a.q_tiles * a.chunks;
    if (ctas > INT32_MAX) return fail(ANN_ENOTSUP, "attentionScores: grid too large.");
    CUtensorMap smap{}, kmap{};
    ANN_TRY(map_bhtk(a.s, bhs / a.Hq, a.Hq, a.Tq, a.Tk, a.s_b, a.s_h, a.s_t, 32, &smap, "attentionScores"));
    ANN_TRY(map_f32_4d(&kmap, a.k, kdims, kstr, 32, C::KROWS, "attentionScores"));
    return cluster_launch(scores_pair_kernel<D>, kThreads, C::SMEM, ctas, stream, "attentionScores (tensor cores)", a,
                          smap, kmap);
}

template <int D>
int launch_apply(ann_stream stream, ApArgs& a, int64_t bhs, bool can_split, void* out_zero, size_t out_bytes) {
    using C = ApCfg<D>;
    CUtensorMap pmap{};
    ANN_TRY(map_bhtk(a.p, bhs / a.Hq, a.Hq, a.Tq, a.Tk, a.p_b, a.p_h, a.p_t, kBM, &pmap, "attentionApply"));
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(apply_pair_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    if (attr != cudaSuccess) return fail(ANN_ECUDA, "attentionApply (tensor cores) setup: %s", cudaGetErrorString(attr));
    int64_t const units = bhs * a.q_tiles, slots = sm_count() / 2;
    // two key halves when one unit per tile would leave a short grid
    a.splits = (can_split && units < 3 * slots && a.chunks >= 16) ? 2 : 1;
    if (a.splits == 2) {
        cudaError_t const e = cudaMemsetAsync(out_zero, 0, out_bytes, as_stream(stream));
        if (e != cudaSuccess) return fail(ANN_ECUDA, "attentionApply: %s", cudaGetErrorString(e));
    }
    int64_t const ctas = 2 * units * a.splits;
    if (ctas > INT32_MAX) return fail(ANN_ENOTSUP, "attentionApply: grid too large.");
    return cluster_launch(apply_pair_kernel<D>, kApThreads, C::SMEM, ctas, stream, "attentionApply (tensor cores)", a,
                          pmap);
}

bool rows16(const Dims& d, int unit_axis) {  // unit stride on `unit_axis`, 16-byte aligned rows
    if (d.str[unit_axis] != 1 || !aligned(d.data, 16)) return false;
    for (int i = 0; i < d.rank; ++i)
        if (i != unit_axis && d.str[i] % 4 != 0) return false;
    return true;
}

}  // namespace

// fp32 attentionScores on the tensor cores when the shapes allow it (D 64 /
// 128, unit-stride 16-byte aligned rows of Q, K and S, Tk a multiple of 4);
// `handled` = false otherwise (the caller runs the FP32-pipe kernel).
int scores_tc_f32(ann_stream stream, const Dims& q, const Dims& k, const Dims& s, uint32_t g, int layout,
                  bool& handled) {
    handled = false;
    if (tc_disabled()) return ANN_OK;
    int const tok = layout == ANN_LAYOUT_BTHD ? 1 : 2, head = layout == ANN_LAYOUT_BTHD ? 2 : 1;
    int64_t const B = s.ext[0], Hq = s.ext[1], Tq = s.ext[2], Tk = s.ext[3], D = q.ext[3];
    if ((D != 64 && D != 128) || Tk % 4 != 0 || Tq < 1 || Tk < 1) return ANN_OK;
    if (!rows16(q, 3) || !rows16(k, 3) || !rows16(s, 3) || !tma_view(s)) return ANN_OK;
    int64_t const kdims[4] = {k.ext[3], k.ext[tok], k.ext[head], k.ext[0]};  // K as (d, key, head, batch)
    int64_t const kstr[3] = {k.str[tok], k.str[head], k.str[0]};
    if (!tma_view_ok(kdims, kstr)) return ANN_OK;
    ScArgs a{};
    a.q = static_cast<const float*>(q.data);
    a.k = static_cast<const float*>(k.data);
    a.s = static_cast<float*>(s.data);
    a.q_b = q.str[0];
    a.q_t = q.str[1];
    a.q_h = q.str[2];
    a.k_b = k.str[0];
    a.k_t = k.str[tok];
    a.k_h = k.str[head];
    a.s_b = s.str[0];
    a.s_h = s.str[1];
    a.s_t = s.str[2];
    a.Tq = Tq;
    a.Tk = Tk;
    a.Hq = Hq;
    a.g = g;
    int64_t const q_tiles = ceil_div(Tq, 2 * kBM), k_tiles = ceil_div(Tk, ScCfg<64>::NT);
    if (q_tiles > INT32_MAX || k_tiles > INT32_MAX) return ANN_OK;
    a.q_tiles = static_cast<int>(q_tiles);
    a.k_tiles = static_cast<int>(k_tiles);
    handled = true;
    return D == 64 ? launch_scores<64>(stream, a, B * Hq, kdims, kstr)
                   : launch_scores<128>(stream, a, B * Hq, kdims, kstr);
}

// fp32 attentionApply on the tensor cores (D 64 / 128, unit-stride 16-byte
// aligned rows of P, V and out, Tk a multiple of 4); `handled` as above.
int apply_tc_f32(ann_stream stream, const Dims& p, const Dims& v, const Dims& o, uint32_t g, int layout,
                 bool& handled) {
    handled = false;
    if (tc_disabled()) return ANN_OK;
    int const tok = layout == ANN_LAYOUT_BTHD ? 1 : 2, head = layout == ANN_LAYOUT_BTHD ? 2 : 1;
    int64_t const B = o.ext[0], Tq = o.ext[1], Hq = o.ext[2], D = o.ext[3], Tk = p.ext[3];
    if ((D != 64 && D != 128) || Tk % 4 != 0 || Tq < 1 || Tk < 1) return ANN_OK;
    if (!rows16(p, 3) || !rows16(v, 3) || !rows16(o, 3)) return ANN_OK;
    if (!tma_view(p)) return ANN_OK;
    ApArgs a{};
    a.p = static_cast<const float*>(p.data);
    a.v = static_cast<const float*>(v.data);
    a.o = static_cast<float*>(o.data);
    a.p_b = p.str[0];
    a.p_h = p.str[1];
    a.p_t = p.str[2];
    a.v_b = v.str[0];
    a.v_t = v.str[tok];
    a.v_h = v.str[head];
    a.o_b = o.str[0];
    a.o_t = o.str[1];
    a.o_h = o.str[2];
    a.Tq = Tq;
    a.Tk = Tk;
    a.Hq = Hq;
    a.g = g;
    int64_t const q_tiles = ceil_div(Tq, 2 * kBM);
    if (q_tiles > INT32_MAX) return ANN_OK;
    a.q_tiles = static_cast<int>(q_tiles);
    a.chunks = ceil_div(Tk, static_cast<int64_t>(ApCfg<64>::KC));
    // the split adds into a zeroed output: only for a dense output tensor
    bool const dense = o.dense();
    size_t const out_bytes = static_cast<size_t>(o.numel()) * 4;
    handled = true;
    return D == 64 ? launch_apply<64>(stream, a, B * Hq, dense, o.data, out_bytes)
                   : launch_apply<128>(stream, a, B * Hq, dense, o.data, out_bytes);
}

int take_attention_tc_error(cudaStream_t s, uint32_t* bits) {
    unsigned int value = 0, zero = 0;
    if (cudaMemcpyFromSymbolAsync(&value, g_atc_error, sizeof value, 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_atc_error, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ANN_ECUDA, "device error word: %s", cudaGetErrorString(cudaGetLastError()));
    *bits |= value;
    return ANN_OK;
}

}  // namespace ann
