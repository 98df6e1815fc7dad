// prefill_tc.cu -- fp32 fused prefill attention on the sm_100a tensor cores (tcgen05), 3xTF32.
//
// Same pipeline and semantics as prefill.cu (attentionScores -> ops::scale ->
// causalSoftmax with the top-left mask / softmax -> attentionApply, reference
// test/unit/nn/attention.cpp:591-651), with both contractions on tcgen05.mma
// kind::tf32 and fp32 accuracy kept by the 3xTF32 split x = hi + lo, each
// product taken as hi*hi + hi*lo + lo*hi (the dropped lo*lo term is ~2^-21
// relative). A kind::tf32 MMA reads an fp32 operand by dropping its low 13
// mantissa bits, so the raw fp32 value serves as hi as it stands and only
// lo = x - trunc13(x) (exact in fp32, truncated again by the MMA) is computed.
//
// One CTA owns 128 query rows of one (batch, head) and walks its keys in tiles
// of 64, with two warp roles:
//   warps 0..7  two threads per query row (TMEM lane r = tid % 128, half
//               h = tid / 128): Q -> TMEM; per tile S(t) -> registers (both
//               halves load the whole row and take its max, so no exchange is
//               needed), K(t+2) -> shared memory, online softmax with a lazy
//               rescale (O and l are rescaled only when the running max grows by
//               more than 8 in natural-log units, exact because O and l share
//               the max used) over the half's 32 keys, V(t) -> shared memory,
//               P_hi -> TMEM, P_lo -> shared memory, O rescale of the half's D/2
//               columns. K and V go global -> registers one tile ahead ->
//               shared memory as hi (raw) and lo, in the layouts the MMA reads
//               (K: K-major, 128-byte swizzle; V: MN-major, 128-byte swizzle of
//               32-byte chunks).
//   warp 8      one thread issues the S = Q K^T MMAs
//   warp 9      one thread issues the O += P V MMAs
//               (two issuers: a single thread cannot issue MMAs as fast as the
//               tensor pipe runs them; S and PV touch disjoint TMEM columns and
//               complete on their own mbarriers through tcgen05.commit)
//   TMEM  [Q_hi | Q_lo | O | S (64) | P_hi (64)]   = 512 columns for D = 128
//   smem  K hi/lo x 2 buffers | V hi/lo | P_lo     = 224 KB for D = 128
// S(t+1) runs alongside PV(t); the softmax of tile t and the V split run while
// S(t+1) and PV(t-1) execute. Per 64-key tile the MMAs
// are S: 3 x D/8 of M128 N64 K8 (A = Q from TMEM) and PV: 3 x 8 of M128 N=D K8
// (A = P_hi from TMEM, P_lo from shared memory).
// Every wait is bounded; on a timeout the CTA stops, waits for its issued MMAs,
// frees its TMEM and reports ANN_DEVERR_WAIT_TIMEOUT.
#include <cstdlib>
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

constexpr int kBM = 128, kBN = 64;
constexpr int kRowThreads = 256;  // warps 0..7
constexpr int kThreads = kRowThreads + 64;  // + warp 8 (S issuer) and warp 9 (PV issuer)
constexpr float kLog2e = 1.44269504088896341f;
constexpr float kLazy2 = 8.0f * kLog2e;  // lazy-rescale threshold, log2 units

template <int D>
struct TcCfg {
    static constexpr int TILE = kBN * D * 4;  // bytes of one K or V tile (hi or lo)
    static constexpr int BLK = kBN * 128;     // one 32-float column block of a tile: 64 rows x 128 B
    static constexpr int OFF_K = 0;           // buffer i: hi at OFF_K + 2*i*TILE, lo at + TILE
    static constexpr int OFF_V = 4 * TILE;    // hi, lo
    static constexpr int OFF_PLO = 6 * TILE;  // P_lo: 128 rows x 64 keys as two 32-key blocks
    static constexpr int PLO_BLK = kBM * 128;
    static constexpr int OFF_BAR = OFF_PLO + 2 * PLO_BLK;
    // barriers: qready kready[2] vready sfull sfree pfull pvdone drain_s drain_pv
    static constexpr int NBAR = 10;
    static constexpr int OFF_SLOT = OFF_BAR + NBAR * 8;  // TMEM base, abort flag
    static constexpr int USED = OFF_SLOT + 16;
    // + 1 KB to align the base to the 1 KB swizzle atom; >= 120 KB so that a
    // single CTA is resident per SM (it allocates all 512 TMEM columns)
    static constexpr int SMEM = USED + 1024 > 120 * 1024 ? USED + 1024 : 120 * 1024;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    // TMEM columns
    static constexpr uint32_t Q_HI = 0, Q_LO = D, O_COL = 2 * D, S_COL = 3 * D, P_HI = 3 * D + kBN;
    static constexpr uint32_t TMEM_COLS = 512;
    static_assert(P_HI + kBN <= TMEM_COLS, "TMEM budget");
    static constexpr uint32_t IDESC_S = tc::idesc_tf32(kBM, kBN, false);
    static constexpr uint32_t IDESC_PV = tc::idesc_tf32(kBM, D, true);
};

struct TcArgs {
    void* out;
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
    int o_vec;  // out rows are unit-stride and 16-byte aligned
    int q_tiles;
    int64_t bhs;         // batch * query heads
    int64_t head_chunk;  // (batch, head) pairs per dispatch chunk
};

// lo part of the 3xTF32 split: hi is x itself (a kind::tf32 MMA reads an fp32
// operand by dropping its low 13 mantissa bits), lo = x - trunc13(x) is exact
// and is in turn truncated to tf32 by the MMA, so each product keeps a relative
// error below 2^-19 (hi*lo and lo*hi to 2^-20 each, the dropped lo*lo 2^-20).
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

__device__ __forceinline__ void row_sync() {  // the 256 row threads (warps 0..7)
    asm volatile("bar.sync 1, %0;" ::"n"(kRowThreads) : "memory");
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(TcArgs a, float scale) {
    using C = TcCfg<D>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    uint32_t const raw_base = smem_u32(smem_raw);
    uint32_t const pad = (1024u - (raw_base & 1023u)) & 1023u;
    unsigned char* smem = smem_raw + pad;
    uint32_t const sbase = raw_base + pad;
    uint32_t const bar = sbase + C::OFF_BAR;
    uint32_t const qready = bar, kready = bar + 8, vready = bar + 24, sfull = bar + 32, sfree = bar + 40,
                   pfull = bar + 48, pvdone = bar + 56, drain_s = bar + 64, drain_pv = bar + 72;
    uint32_t* slot = reinterpret_cast<uint32_t*>(smem + C::OFF_SLOT);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + C::OFF_SLOT + 4);

    int const tid = threadIdx.x, warp = tid >> 5;
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
    int64_t const k_end = a.causal ? (a.Tk < q0 + kBM ? a.Tk : q0 + kBM) : a.Tk;
    int const n_kt = static_cast<int>((k_end + kBN - 1) / kBN);

    if (tid == 0) {
        mbar_init(qready, kRowThreads);
        for (int i = 0; i < 2; ++i) mbar_init(kready + 8 * i, kRowThreads);
        mbar_init(vready, kRowThreads);
        mbar_init(sfull, 1);
        mbar_init(sfree, kRowThreads);
        mbar_init(pfull, kRowThreads);
        mbar_init(pvdone, 1);
        mbar_init(drain_s, 1);
        mbar_init(drain_pv, 1);
        fence_mbar_init();
        *abort = 0;
    }
    if (warp == 0) {
        tc::tmem_alloc(smem_u32(slot), C::TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    uint32_t const tmem = *slot;

    if (warp >= 8) {
        // ============================== MMA issue (8, 9) ==============================
        if ((tid & 31) == 0) {
            // Descriptors are built once; a tile or k-step offset is added to the
            // 14-bit start-address field (all of shared memory is < 2^18 bytes,
            // so the field never carries).
            uint64_t const k_desc = tc::smem_desc(sbase + C::OFF_K, 16, 1024, tc::kSwizzle128B);
            uint64_t const v_desc = tc::smem_desc(sbase + C::OFF_V, C::BLK, 512, tc::kSwizzle128B_32B);
            uint64_t const p_desc = tc::smem_desc(sbase + C::OFF_PLO, 16, 1024, tc::kSwizzle128B);
            auto at = [](uint64_t desc, uint32_t off) { return desc + static_cast<uint64_t>(off >> 4); };
            auto issue_s = [&](int t) {  // S = Q K^T (tile t)
                uint32_t const kb = static_cast<uint32_t>(t & 1) * 2 * C::TILE;
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk) {
                    uint32_t const off = kb + (kk >> 2) * C::BLK + (kk & 3) * 32;
                    uint64_t const khi = at(k_desc, off), klo = at(k_desc, off + C::TILE);
                    tc::mma_tf32_ts(tmem + C::S_COL, tmem + C::Q_HI + 8 * kk, khi, C::IDESC_S, kk > 0 ? 1u : 0u);
                    tc::mma_tf32_ts(tmem + C::S_COL, tmem + C::Q_HI + 8 * kk, klo, C::IDESC_S, 1u);
                    tc::mma_tf32_ts(tmem + C::S_COL, tmem + C::Q_LO + 8 * kk, khi, C::IDESC_S, 1u);
                }
                tc::mma_commit(sfull);
            };
            auto issue_pv = [&](int t) {  // O += P V (tile t)
#pragma unroll
                for (int kk = 0; kk < kBN / 8; ++kk) {
                    uint64_t const vhi = at(v_desc, kk * 1024), vlo = at(v_desc, C::TILE + kk * 1024);
                    uint64_t const plo = at(p_desc, (kk >> 2) * C::PLO_BLK + (kk & 3) * 32);
                    tc::mma_tf32_ts(tmem + C::O_COL, tmem + C::P_HI + 8 * kk, vhi, C::IDESC_PV,
                                    (t > 0 || kk > 0) ? 1u : 0u);
                    tc::mma_tf32_ts(tmem + C::O_COL, tmem + C::P_HI + 8 * kk, vlo, C::IDESC_PV, 1u);
                    tc::mma_tf32_ss(tmem + C::O_COL, plo, vhi, C::IDESC_PV, 1u);
                }
                tc::mma_commit(pvdone);
            };
            if (warp == 8) {  // S(t) once K(t) is stored and softmax(t-1) has read S(t-1)
                bool ok = n_kt == 0 || mbar_wait_or_abort(qready, 0, abort);
                for (int t = 0; t < n_kt && ok; ++t) {
                    ok = mbar_wait_or_abort(kready + 8 * (t & 1), (t >> 1) & 1, abort) &&
                         (t == 0 || mbar_wait_or_abort(sfree, (t - 1) & 1, abort));
                    if (!ok) break;
                    tc::fence_after_sync();
                    issue_s(t);
                }
            } else {  // PV(t) once P(t) and V(t) are in place
                for (int t = 0; t < n_kt; ++t) {
                    bool const ok = mbar_wait_or_abort(pfull, t & 1, abort) && mbar_wait_or_abort(vready, t & 1, abort);
                    if (!ok) break;
                    tc::fence_after_sync();
                    issue_pv(t);
                }
            }
            // every MMA this thread issued has finished reading TMEM and shared
            // memory before either is released
            uint32_t const drain = warp == 8 ? drain_s : drain_pv;
            tc::mma_commit(drain);
            if (!mbar_wait_bounded(drain, 0)) *abort = 1;
        }
    } else {
        // ============================ row warps (0..7) ============================
        int const r = tid & (kBM - 1), h = tid >> 7;
        uint32_t const lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
        int64_t const qi = q0 + r;
        constexpr int HD = D / 2;  // O / Q columns per half

        // ---- K / V tiles: element e = i * 256 + tid is key row e / NV4, float4 column e % NV4
        constexpr int NV4 = D / 4;
        constexpr int PER = kBN * NV4 / kRowThreads;  // float4 per thread per tile
        float const* kbase = a.k + b * a.k_b + kvh * a.k_h;
        float const* vbase = a.v + b * a.v_b + kvh * a.v_h;
        float4 rk[PER], rv[PER];
        auto load = [&](float4 (&rg)[PER], float const* base, int64_t stride_t, int t) {
#pragma unroll
            for (int i = 0; i < PER; ++i) {
                int const e = i * kRowThreads + tid, row = e / NV4, c4 = e % NV4;
                int64_t const key = static_cast<int64_t>(t) * kBN + row;
                rg[i] = key < a.Tk ? __ldg(reinterpret_cast<float4 const*>(base + key * stride_t) + c4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);  // V rows past Tk must be finite
            }
        };
        auto store_k = [&](float4 const (&rg)[PER], int buf) {  // K-major, 16-byte chunks XOR (row % 8)
            unsigned char* hi = smem + C::OFF_K + buf * 2 * C::TILE;
#pragma unroll
            for (int i = 0; i < PER; ++i) {
                int const e = i * kRowThreads + tid, row = e / NV4, c4 = e % NV4;
                int const off = (c4 >> 3) * C::BLK + row * 128 + (((c4 & 7) ^ (row & 7)) << 4);
                *reinterpret_cast<float4*>(hi + off) = rg[i];
                *reinterpret_cast<float4*>(hi + C::TILE + off) = tf32_lo(rg[i]);
            }
            tc::fence_proxy_async_smem();  // visible to the tensor core
        };
        auto store_v = [&](float4 const (&rg)[PER]) {  // MN-major, 32-byte chunks XOR (row % 4)
            unsigned char* hi = smem + C::OFF_V;
#pragma unroll
            for (int i = 0; i < PER; ++i) {
                int const e = i * kRowThreads + tid, row = e / NV4, c4 = e % NV4;
                int const off =
                    (c4 >> 3) * C::BLK + row * 128 + ((((c4 & 7) >> 1) ^ (row & 3)) << 5) + ((c4 & 1) << 4);
                *reinterpret_cast<float4*>(hi + off) = rg[i];
                *reinterpret_cast<float4*>(hi + C::TILE + off) = tf32_lo(rg[i]);
            }
            tc::fence_proxy_async_smem();
        };
        if (n_kt > 0) {
            load(rk, kbase, a.k_t, 0);
            load(rv, vbase, a.v_t, 0);
        }
        {  // Q row half -> TMEM: hi (raw) and lo, the A operand of S = Q K^T
            float const* qrow = a.q + b * a.q_b + qi * a.q_t + hq * a.q_h + h * HD;
            bool const live = qi < a.Tq;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                float hi[32], lo[32];
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    float4 const x = live ? __ldg(reinterpret_cast<float4 const*>(qrow + 32 * c + j))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
                    hi[j] = x.x, hi[j + 1] = x.y, hi[j + 2] = x.z, hi[j + 3] = x.w;
                    lo[j] = tf32_lo(x.x), lo[j + 1] = tf32_lo(x.y), lo[j + 2] = tf32_lo(x.z),
                    lo[j + 3] = tf32_lo(x.w);
                }
                tc::tmem_st32(tmem + lane_off + C::Q_HI + h * HD + 32 * c, hi);
                tc::tmem_st32(tmem + lane_off + C::Q_LO + h * HD + 32 * c, lo);
            }
            tc::tmem_st_wait();
            tc::fence_before_sync();
            mbar_arrive(qready);
        }
        // K runs two tiles ahead: K(0), K(1) now; K(t+2) into buffer t % 2 as soon
        // as S(t) has landed, so that S(t+1) waits only for softmax(t) to read S(t)
        for (int t = 0; t < (n_kt < 2 ? n_kt : 2); ++t) {
            if (t == 1) load(rk, kbase, a.k_t, 1);
            store_k(rk, t);
            mbar_arrive(kready + 8 * t);
        }
        if (n_kt > 2) load(rk, kbase, a.k_t, 2);
        unsigned char* plo_row = smem + C::OFF_PLO + h * C::PLO_BLK + r * 128;
        float const c2 = scale * kLog2e;  // scores are taken in log2 units: s * scale * log2(e)
        float m_used = Lowest<float>::value, l_part = 0.f;
        bool ok = true;
        // Decisions after a wait are made warp-uniform (__all_sync): tcgen05.ld/st
        // are warp-collective, so a warp must never split on an abort.
        for (int t = 0; t < n_kt && ok; ++t) {
            ok = __all_sync(0xffffffffu, mbar_wait_or_abort(sfull, t & 1, abort));
            if (!ok) break;  // S(t) done: K buffer t % 2 is free
            tc::fence_after_sync();
            float sv[kBN];  // [0, 32): this half's keys, [32, 64): the other half's
            tc::tmem_ld32x2(tmem + lane_off + C::S_COL + 32 * h, tmem + lane_off + C::S_COL + 32 * (1 - h), sv);
            tc::fence_before_sync();
            mbar_arrive(sfree);  // S(t+1) may overwrite the accumulator
            if (t + 2 < n_kt) {
                store_k(rk, t & 1);  // K(t+2)
                mbar_arrive(kready + 8 * (t & 1));
                if (t + 3 < n_kt) load(rk, kbase, a.k_t, t + 3);
            }
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
            mbar_arrive(pfull);
            store_v(rv);
            mbar_arrive(vready);
            if (t + 1 < n_kt) load(rv, vbase, a.v_t, t + 1);
        }
        if (ok && n_kt > 0) ok = mbar_wait_or_abort(pvdone, (n_kt - 1) & 1, abort);
        ok = __all_sync(0xffffffffu, ok);
        // row sum = the two halves' parts, exchanged through the (now idle) P_lo
        // buffer; every row thread reaches this barrier exactly once
        float* lx = reinterpret_cast<float*>(smem + C::OFF_PLO);
        if (ok) lx[tid] = l_part;
        row_sync();
        if (ok) {
            tc::fence_after_sync();
            float const l_sum = lx[r] + lx[r + kBM];
            float const inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
            float* orow = static_cast<float*>(a.out) + b * a.o_b + qi * a.o_t + hq * a.o_h;
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
                        for (int j = 0; j < 32; ++j) orow[(col + j) * a.o_d] = ov[j] * inv;
                    }
                }
            }
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (*abort && tid == 0) atomicOr(&g_tc_error, ANN_DEVERR_WAIT_TIMEOUT);
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int D>
int launch_tc(ann_stream stream, const Dims& q, const Dims& k, const Dims& v, const Dims& o, float scale, uint32_t g,
              int layout, int causal, bool& handled) {
    using C = TcCfg<D>;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(prefill_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    if (attr != cudaSuccess)
        return fail(ANN_ECUDA, "attention prefill (tensor cores) setup: %s", cudaGetErrorString(attr));
    int const tok = layout == ANN_LAYOUT_BTHD ? 1 : 2, head = layout == ANN_LAYOUT_BTHD ? 2 : 1;
    TcArgs a{};
    a.out = o.data;
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
              o.str[1] % 4 == 0 && o.str[2] % 4 == 0;
    a.Tq = q.ext[1];
    a.Tk = k.ext[tok];
    a.Hq = q.ext[2];
    a.g = g;
    a.causal = causal;
    int64_t const q_tiles = ceil_div(a.Tq, kBM);
    int64_t const bhs = q.ext[0] * q.ext[2];
    if (q_tiles * bhs > INT32_MAX) return ANN_OK;  // not handled
    a.q_tiles = static_cast<int>(q_tiles);
    handled = true;
    a.bhs = bhs;
    a.head_chunk = head_chunk_for(bhs, q_tiles, 2 * a.Tk * q.ext[3] * 4, 1);
    dim3 grid(static_cast<unsigned>(q_tiles * bhs));
    prefill_tc_kernel<D><<<grid, kThreads, C::SMEM, as_stream(stream)>>>(a, scale);
    return check_launch("attention prefill (tensor cores)");
}

}  // namespace

// Runs the tensor-core kernel for fp32 with D 64 or 128 (the caller has checked
// unit-stride, 16-byte aligned Q/K/V rows); sets `handled` = false otherwise.
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
