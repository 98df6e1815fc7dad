// prefill_f64.cu -- fp64 fused prefill attention on the FP64 tensor cores (DMMA).
//
// Same pipeline and semantics as prefill.cu (attentionScores -> ops::scale ->
// causalSoftmax with the top-left mask / softmax -> attentionApply, reference
// test/unit/nn/attention.cpp:591-651), with both contractions as
// mma.sync.m16n8k4.f64 (fp64 products, fp64 accumulation).
//
// One CTA = 64 query rows of one (batch, head), 4 warps of 16 rows; K/V tiles of
// 32 (or 16, see FCfg) keys stream through two shared-memory stages filled by 1-D bulk copies,
// rows padded by 16 bytes (pitch = 16 mod 128 bytes), which makes every
// fragment read below hit each bank at most twice per 256 bytes.
// Fragment layout of m16n8k4.f64 (g = lane / 4, t = lane % 4):
//   A 16x4: a0 = A[g][t], a1 = A[g+8][t];  B 4x8: b0 = B[t][g];
//   C 16x8: c0 = C[g][2t], c1 = C[g][2t+1], c2 = C[g+8][2t], c3 = C[g+8][2t+1].
// S = Q K^T: per k-step of 4 head dims, a0/a1 from Q in shared memory and b0 =
// K[8j + g][4kk + t]. P V without moving P: the MMA may add the keys in any
// order as long as A and B agree, so the k-steps of key block j take keys
// (8j + 2t) and then (8j + 2t + 1) -- exactly the keys thread t already holds
// in its S registers -- with b0 = V[8j + 2t (+1)][8n + g].
// The online softmax (exact rescale every tile) reduces a row over the 4
// threads of a quad with two shuffles.
#include <cooperative_groups.h>

#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "multimem.cuh"
#include "reduce.cuh"
#include "tma.cuh"

namespace ann {

int prefill_mma_f64(ann_stream stream, const Dims& q, const Dims& k, const Dims& v, const Dims& o, double scale,
                    uint32_t g, int layout, int causal, bool& handled, void* mirror);
int take_prefill_f64_error(cudaStream_t s, uint32_t* bits);

namespace {

__device__ unsigned int g_f64_error;

constexpr int kBM = 64, kThreads = 128;

// BN keys per tile. D = 64 with 16-key tiles needs 158 registers and 68 KB of
// shared memory, room for 3 CTAs (12 warps) per SM that keep the DMMA pipe
// fed on long grids; with 32-key tiles (2 CTAs per SM) half as many tiles carry
// the per-tile softmax cost, which wins on short grids (launch_f64 picks).
// D = 128: 32-key tiles, one CTA per SM.
template <int D, int BN_ = 32>
struct FCfg {
    static constexpr int BN = BN_;
    static constexpr int MIN_CTAS = D <= 64 ? (BN <= 16 ? 3 : 2) : 1;
    static constexpr int LD = D + 2;  // row pitch in doubles: 16 bytes of padding
    static constexpr int ROWB = D * 8;
    static constexpr size_t TILE = static_cast<size_t>(BN) * LD;  // doubles per K or V stage
    static constexpr size_t OFF_Q = 0;
    static constexpr size_t OFF_K = OFF_Q + static_cast<size_t>(kBM) * LD * 8;
    static constexpr size_t OFF_V = OFF_K + 2 * TILE * 8;
    static constexpr size_t OFF_BAR = OFF_V + 2 * TILE * 8;
    static constexpr size_t SMEM = OFF_BAR + 3 * sizeof(uint64_t);
    static_assert((LD * 8) % 128 == 16, "row pitch = 16 mod 128 bytes");
};

struct F64Args {
    const double* q;
    const double* k;
    const double* v;
    double* out;
    double* mirror;  // multicast address of out[0] (every O store goes to all ranks' copies), or null
    int64_t q_b, q_t, q_h;
    int64_t o_b, o_t, o_h, o_d;
    int64_t k_b, k_h, k_t;
    int64_t v_b, v_h, v_t;
    int64_t Tq, Tk, Hq;
    uint32_t g;
    int causal;
    int o_pairs;  // out rows unit-stride and 16-byte aligned: store pairs
    int q_tiles;
    int64_t bhs;         // batch * query heads
    int64_t head_chunk;  // (batch, head) pairs per dispatch chunk
    int splits;          // CTAs (one cluster) sharing the key range of one query tile: 1, 2 or 4
};

__device__ __forceinline__ void dmma(double (&c)[4], double a0, double a1, double b0) {
    asm volatile("mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
                 : "d"(a0), "d"(a1), "d"(b0));
}

__device__ __forceinline__ double quad_max(double x) {
    x = fmax(x, __shfl_xor_sync(0xffffffffu, x, 1));
    return fmax(x, __shfl_xor_sync(0xffffffffu, x, 2));
}
__device__ __forceinline__ double quad_sum(double x) {
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    return x + __shfl_xor_sync(0xffffffffu, x, 2);
}

// Merge of the key-range splits of one query tile (a cluster of a.splits CTAs):
// each CTA leaves its unnormalised O, row max and row sum in its own shared
// memory (the K/V stages, drained by now), then CTA s combines rows
// [64 s / S, 64 (s + 1) / S) of all partials through distributed shared memory
// with the log-sum-exp rule O = sum_s O_s e^(m_s - M) / sum_s l_s e^(m_s - M),
// M = max_s m_s, and stores them. The second cluster barrier keeps every CTA's
// shared memory alive until its peers have read it.
template <int D>
__device__ void merge_splits(F64Args const& a, unsigned char* smem, double const (&o)[D / 8][4],
                             double const (&m_run)[2], double const (&l_run)[2], int q_rows, int64_t b, int64_t hq,
                             int64_t q0) {
    namespace cg = cooperative_groups;
    constexpr int NO = D / 8;
    constexpr int LDP = D + 1;  // partial O row pitch in doubles
    int const tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int const g = lane >> 2, t = lane & 3;
    int const r0 = 16 * warp + g;
    // [kBM][LDP] O, then m[kBM], l[kBM], over the Q tile and the K/V stages (all
    // free now; they hold more than this for every tile size)
    double* part = reinterpret_cast<double*>(smem);
    // smallest layout (16-key tiles): Q (kBM rows) + four 16-row K/V stages of D + 2 doubles
    static_assert((kBM * (D + 1) + 2 * kBM) * 8 <= (kBM + 4 * 16) * (D + 2) * 8, "merge buffer fits");
    double* pm = part + kBM * LDP;
    double* pl = pm + kBM;
    __syncthreads();  // every warp is done with the K/V stages
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        int const r = r0 + 8 * h;
#pragma unroll
        for (int n = 0; n < NO; ++n) {
            part[r * LDP + 8 * n + 2 * t] = o[n][2 * h];
            part[r * LDP + 8 * n + 2 * t + 1] = o[n][2 * h + 1];
        }
        if (t == 0) {
            pm[r] = m_run[h];
            pl[r] = l_run[h];
        }
    }
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    int const S = a.splits, s = static_cast<int>(cluster.block_rank());
    int const row_lo = kBM * s / S, row_hi = kBM * (s + 1) / S;
    for (int e = tid; e < (row_hi - row_lo) * D; e += kThreads) {
        int const r = row_lo + e / D, c = e % D;
        if (r >= q_rows) continue;
        double M = Lowest<double>::value;
        for (int p = 0; p < S; ++p) M = fmax(M, cluster.map_shared_rank(pm, p)[r]);
        double L = 0.0, acc = 0.0;
        for (int p = 0; p < S; ++p) {
            double const w = exp(cluster.map_shared_rank(pm, p)[r] - M);
            L += w * cluster.map_shared_rank(pl, p)[r];
            acc += w * cluster.map_shared_rank(part, p)[r * LDP + c];
        }
        double const val = L > 0.0 ? acc / L : 0.0;
        int64_t const off = b * a.o_b + (q0 + r) * a.o_t + hq * a.o_h + c * a.o_d;
        if (a.mirror) mc::store(a.mirror + off, val);
        else a.out[off] = val;
    }
    cluster.sync();
}

template <int D, int BN>
__global__ void __launch_bounds__(kThreads, FCfg<D, BN>::MIN_CTAS) prefill_f64_kernel(F64Args a, double scale) {
    using C = FCfg<D, BN>;
    constexpr int kBN = C::BN;
    constexpr int NJ = kBN / 8;  // key blocks of 8 per tile
    constexpr int NO = D / 8;    // output column blocks of 8
    extern __shared__ __align__(128) unsigned char smem[];
    double* Qs = reinterpret_cast<double*>(smem + C::OFF_Q);
    double* Ks = reinterpret_cast<double*>(smem + C::OFF_K);
    double* Vs = reinterpret_cast<double*>(smem + C::OFF_V);
    uint32_t const bar0 = smem_u32(smem + C::OFF_BAR);  // [0] Q, [1] stage 0, [2] stage 1

    int const tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int const g = lane >> 2, t = lane & 3;
    // 1-D grid in chunks of a.head_chunk (batch, head) pairs (head_chunk_for):
    // inside a chunk the query tiles go from the last (most keys) down, so the
    // heaviest CTAs start first, while the K/V of one chunk stay in L2. With
    // a.splits > 1 a cluster of that many CTAs shares one query tile, CTA s
    // taking the s-th contiguous share of its key tiles.
    int const split = static_cast<int>(blockIdx.x % a.splits);
    int64_t const lin = blockIdx.x / a.splits, per_chunk = a.head_chunk * a.q_tiles;
    int64_t const chunk = lin / per_chunk, in_chunk = lin % per_chunk;
    int64_t const chunk_bh = a.bhs - chunk * a.head_chunk < a.head_chunk ? a.bhs - chunk * a.head_chunk : a.head_chunk;
    int const qt = a.q_tiles - 1 - static_cast<int>(in_chunk / chunk_bh);
    int64_t const bh = chunk * a.head_chunk + in_chunk % chunk_bh;
    int64_t const hq = bh % a.Hq, b = bh / a.Hq, kvh = hq / a.g;
    int64_t const q0 = static_cast<int64_t>(qt) * kBM;
    int const q_rows = static_cast<int>(q0 + kBM <= a.Tq ? kBM : a.Tq - q0);
    int64_t const k_end = a.causal ? (a.Tk < q0 + kBM ? a.Tk : q0 + kBM) : a.Tk;
    int const n_all = static_cast<int>((k_end + kBN - 1) / kBN);  // key tiles of this query tile
    int const kt0 = static_cast<int>(static_cast<int64_t>(n_all) * split / a.splits);  // this CTA's share
    int const n_kt = static_cast<int>(static_cast<int64_t>(n_all) * (split + 1) / a.splits) - kt0;
    bool const has_last = kt0 + n_kt == n_all;  // holds the (possibly ragged) last key tile

    double const* qbase = a.q + b * a.q_b + q0 * a.q_t + hq * a.q_h;
    double const* kbase = a.k + b * a.k_b + kvh * a.k_h;
    double const* vbase = a.v + b * a.v_b + kvh * a.v_h;

    auto issue_kv = [&](int kt) {  // warp 0: K and V rows of this CTA's key tile kt into stage kt & 1
        int const s = kt & 1;
        int64_t const key0 = static_cast<int64_t>(kt0 + kt) * kBN;
        int const rows = static_cast<int>(key0 + kBN <= a.Tk ? kBN : a.Tk - key0);
        uint32_t const bar = bar0 + 8 * (1 + s);
        if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(2 * rows * C::ROWB));
        __syncwarp();
        uint32_t const kd = smem_u32(Ks + s * C::TILE), vd = smem_u32(Vs + s * C::TILE);
        for (int r = lane; r < rows; r += 32) {
            bulk_copy_g2s(kd + r * C::LD * 8, kbase + (key0 + r) * a.k_t, C::ROWB, bar);
            bulk_copy_g2s(vd + r * C::LD * 8, vbase + (key0 + r) * a.v_t, C::ROWB, bar);
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
        for (int kt = 0; kt < (n_kt < 2 ? n_kt : 2); ++kt) issue_kv(kt);
    }
    // Q rows past Tq: zeros (never stored). V rows past Tk in the last key tile must
    // be finite (their P is 0, and 0 * NaN is not); K rows there are masked by
    // select. The last tile's stage is zeroed once it is free for that tile.
    for (int i = tid; i < (kBM - q_rows) * C::LD; i += kThreads) Qs[q_rows * C::LD + i] = 0.0;
    int const v_tail = n_kt > 0 && has_last ? static_cast<int>(static_cast<int64_t>(n_all) * kBN - a.Tk) : 0;
    auto zero_v_tail = [&]() {  // all threads; rows [kBN - v_tail, kBN) of the last tile's stage
        double* vt = Vs + ((n_kt - 1) & 1) * C::TILE + (kBN - v_tail) * C::LD;
        for (int i = tid; i < v_tail * C::LD; i += kThreads) vt[i] = 0.0;
    };
    if (v_tail > 0 && n_kt <= 2) zero_v_tail();  // that stage has not been used yet

    int const r0 = 16 * warp + g;  // this thread's rows: r0 and r0 + 8 of the tile
    double m_run[2] = {Lowest<double>::value, Lowest<double>::value}, l_run[2] = {0.0, 0.0};
    double o[NO][4];
#pragma unroll
    for (int n = 0; n < NO; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0;

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
        double const* Kt = Ks + s * C::TILE;
        double const* Vt = Vs + s * C::TILE;
        int64_t const key0 = static_cast<int64_t>(kt0 + kt) * kBN;

        // ---- S = Q K^T: 16 rows x 32 keys per warp
        double sacc[NJ][4];
#pragma unroll
        for (int j = 0; j < NJ; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.0;
#pragma unroll 4
        for (int kk = 0; kk < D / 4; ++kk) {
            double const a0 = Qs[r0 * C::LD + 4 * kk + t], a1 = Qs[(r0 + 8) * C::LD + 4 * kk + t];
#pragma unroll
            for (int j = 0; j < NJ; ++j) dmma(sacc[j], a0, a1, Kt[(8 * j + g) * C::LD + 4 * kk + t]);
        }

        // ---- scale, mask, online softmax (rows r0 and r0 + 8)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int64_t const qi = q0 + r0 + 8 * h;
            double tmax = Lowest<double>::value;
#pragma unroll
            for (int j = 0; j < NJ; ++j)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    int64_t const kj = key0 + 8 * j + 2 * t + e;
                    bool const live = kj < a.Tk && !(a.causal && qi < kj);
                    double const x = sacc[j][2 * h + e] * scale;  // attentionScores, then ops::scale
                    sacc[j][2 * h + e] = live ? x : -INFINITY;
                    if (live) tmax = fmax(tmax, x);
                }
            double const m_new = fmax(m_run[h], quad_max(tmax));
            // rescale only when the row max grew (the same in the 4 threads of a
            // quad): otherwise alpha = exp(0) = 1 and every product by it is exact,
            // so skipping them changes no bit
            bool const grow = m_new != m_run[h];
            double const alpha = grow ? exp(m_run[h] - m_new) : 1.0;
            double psum = 0.0;
#pragma unroll
            for (int j = 0; j < NJ; ++j)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    double const p = exp(sacc[j][2 * h + e] - m_new);  // masked: exp(-inf) = 0
                    sacc[j][2 * h + e] = p;
                    psum += p;
                }
            l_run[h] = (grow ? l_run[h] * alpha : l_run[h]) + quad_sum(psum);
            m_run[h] = m_new;
            if (grow) {
#pragma unroll
                for (int n = 0; n < NO; ++n) {
                    o[n][2 * h] *= alpha;
                    o[n][2 * h + 1] *= alpha;
                }
            }
        }

        // ---- O += P V, P straight from the S registers (keys 8j+2t, then 8j+2t+1)
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                double const* vrow = Vt + (8 * j + 2 * t + e) * C::LD + g;
#pragma unroll
                for (int n = 0; n < NO; ++n) dmma(o[n], sacc[j][e], sacc[j][2 + e], vrow[8 * n]);
            }
        __syncthreads();
        if (kt + 2 == n_kt - 1 && v_tail > 0) zero_v_tail();  // its stage was freed just now
        if (warp == 0 && kt + 2 < n_kt) issue_kv(kt + 2);
    }

    if (!ok) {
        if (tid == 0) {
            atomicOr(&g_f64_error, ANN_DEVERR_WAIT_TIMEOUT);
            for (int kt = abort_kt; kt < (n_kt < abort_kt + 2 ? n_kt : abort_kt + 2); ++kt)  // drain (bounded)
                mbar_wait_bounded(bar0 + 8 * (1 + (kt & 1)), (kt >> 1) & 1);
        }
        if (a.splits > 1) {  // the other CTAs of the cluster still meet at both barriers
            __syncthreads();
            cooperative_groups::this_cluster().sync();
            cooperative_groups::this_cluster().sync();
        }
        return;
    }
    if (a.splits > 1) {
        merge_splits<D>(a, smem, o, m_run, l_run, q_rows, b, hq, q0);
        return;
    }
    if (a.mirror != nullptr && a.o_pairs) {
        // Multicast output: whole rows a warp instruction (512 contiguous bytes,
        // one packet stream to the switch; not 64 bytes from each of 8 rows),
        // staged in the Q tile, which no MMA reads any more. No system-scope
        // fence: the signal barrier after the kernel fences. (Local outputs keep
        // the direct stores below: staging them measured no faster on c4.)
        __syncthreads();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            double const inv = l_run[h] > 0.0 ? 1.0 / l_run[h] : 0.0;
#pragma unroll
            for (int n = 0; n < NO; ++n)
                *reinterpret_cast<double2*>(Qs + (r0 + 8 * h) * C::LD + 8 * n + 2 * t) =
                    make_double2(o[n][2 * h] * inv, o[n][2 * h + 1] * inv);
        }
        __syncthreads();
        constexpr int PAIRS = D / 2;  // double2 per row
        for (int e = tid; e < q_rows * PAIRS; e += kThreads) {
            int const r = e / PAIRS, c2 = e % PAIRS;
            double2 const val = *reinterpret_cast<double2 const*>(Qs + r * C::LD + 2 * c2);
            mc::store(a.mirror + b * a.o_b + (q0 + r) * a.o_t + hq * a.o_h + 2 * c2, val);
        }
        return;
    }
    int64_t const obase_off = b * a.o_b + q0 * a.o_t + hq * a.o_h;
    double* obase = a.out + obase_off;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        int const r = r0 + 8 * h;
        if (r >= q_rows) continue;
        double const inv = l_run[h] > 0.0 ? 1.0 / l_run[h] : 0.0;
        double* orow = obase + r * a.o_t;
        double* mrow = a.mirror ? a.mirror + obase_off + r * a.o_t : nullptr;
#pragma unroll
        for (int n = 0; n < NO; ++n) {
            int const d = 8 * n + 2 * t;
            double const x0 = o[n][2 * h] * inv, x1 = o[n][2 * h + 1] * inv;
            if (mrow) {
                if (a.o_pairs) {
                    mc::store(mrow + d, make_double2(x0, x1));
                } else {
                    mc::store(mrow + d * a.o_d, x0);
                    mc::store(mrow + (d + 1) * a.o_d, x1);
                }
            } else if (a.o_pairs) {
                *reinterpret_cast<double2*>(orow + d) = make_double2(x0, x1);
            } else {
                orow[d * a.o_d] = x0;
                orow[(d + 1) * a.o_d] = x1;
            }
        }
    }
}

template <int D, int BN>
int launch_f64_bn(ann_stream stream, F64Args& a, double scale, int64_t batch_heads) {
    using C = FCfg<D, BN>;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(prefill_f64_kernel<D, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(C::SMEM));
    });
    if (attr != cudaSuccess)
        return fail(ANN_ECUDA, "attention prefill (fp64 MMA) setup: %s", cudaGetErrorString(attr));
    a.bhs = batch_heads;
    a.head_chunk = head_chunk_for(batch_heads, a.q_tiles, 2 * a.Tk * D * 8, C::MIN_CTAS);
    int64_t const ctas = static_cast<int64_t>(a.q_tiles) * batch_heads * a.splits;
    if (a.splits == 1) {
        prefill_f64_kernel<D, BN><<<dim3(static_cast<unsigned>(ctas)), kThreads, C::SMEM, as_stream(stream)>>>(a,
                                                                                                             scale);
        return check_launch("attention prefill (fp64 MMA)");
    }
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute cl{};
    cl.id = cudaLaunchAttributeClusterDimension;
    cl.val.clusterDim.x = static_cast<unsigned>(a.splits);
    cl.val.clusterDim.y = 1;
    cl.val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(ctas));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = as_stream(stream);
    cfg.attrs = &cl;
    cfg.numAttrs = 1;
    cudaError_t const e = cudaLaunchKernelEx(&cfg, prefill_f64_kernel<D, BN>, a, scale);
    if (e != cudaSuccess) return fail(ANN_ECUDA, "attention prefill (fp64 MMA, key splits): %s", cudaGetErrorString(e));
    return check_launch("attention prefill (fp64 MMA, key splits)");
}

// Key-range splits per query tile: 1 while the grid already fills the GPU,
// else 2 or 4, doubling while the CTAs are fewer than two an SM (a
// head-sharded rank's few heads leave most SMs idle, and the last query tiles
// hold every key: without a split they alone set the time). Measured on c4
// (64-row tiles): 256 tiles (the 2-GPU shard) 0.163 ms with 2 splits, 0.202
// with 4, 0.228 with none; 512 tiles (1 GPU) fastest with none (0.236 ms, 0.300
// with 2). ANN_PREFILL_F64_SPLITS pins it.
int f64_splits(int64_t tiles, int max_key_tiles) {
    if (const char* env = std::getenv("ANN_PREFILL_F64_SPLITS")) {
        int const sp = std::atoi(env);
        if (sp == 1 || sp == 2 || sp == 4) return sp;
    }
    int64_t const want = 2 * static_cast<int64_t>(sm_count());
    int sp = 1;
    while (sp < 4 && tiles * sp < want && max_key_tiles >= 4 * sp) sp *= 2;
    return sp;
}

template <int D>
int launch_f64(ann_stream stream, F64Args& a, double scale, int64_t batch_heads) {
    int64_t const tiles = static_cast<int64_t>(a.q_tiles) * batch_heads;
    a.splits = f64_splits(tiles, static_cast<int>(ceil_div(a.causal ? a.Tq : a.Tk, 32)));
    if (tiles * a.splits > INT32_MAX) a.splits = 1;
    if constexpr (D <= 64) {  // ANN_PREFILL_F64_TILE=16 / 32 pins the key tile
        if (const char* env = std::getenv("ANN_PREFILL_F64_TILE")) {
            if (std::atoi(env) == 16) return launch_f64_bn<D, 16>(stream, a, scale, batch_heads);
            if (std::atoi(env) == 32) return launch_f64_bn<D, 32>(stream, a, scale, batch_heads);
        }
    }
    if (a.splits > 1) return launch_f64_bn<D, 32>(stream, a, scale, batch_heads);
    if constexpr (D <= 64) {
        // 16-key tiles once the grid fills at least four waves of 3-CTA slots
        if (static_cast<int64_t>(a.q_tiles) * batch_heads >= int64_t{4} * 3 * sm_count())
            return launch_f64_bn<D, 16>(stream, a, scale, batch_heads);
    }
    return launch_f64_bn<D, 32>(stream, a, scale, batch_heads);
}

}  // namespace

// fp64 prefill on the FP64 tensor cores for D 64 / 128 (the caller has checked
// unit-stride, 16-byte aligned Q/K/V rows); `handled` = false otherwise.
int prefill_mma_f64(ann_stream stream, const Dims& q, const Dims& k, const Dims& v, const Dims& o, double scale,
                    uint32_t g, int layout, int causal, bool& handled, void* mirror) {
    handled = false;
    if (const char* env = std::getenv("ANN_PREFILL_FMA"))
        if (env[0] == '1' && mirror == nullptr) return ANN_OK;
    int64_t const D = q.ext[3];
    if (D != 64 && D != 128) return ANN_OK;
    int const tok = layout == ANN_LAYOUT_BTHD ? 1 : 2, head = layout == ANN_LAYOUT_BTHD ? 2 : 1;
    F64Args a{};
    a.q = static_cast<const double*>(q.data);
    a.k = static_cast<const double*>(k.data);
    a.v = static_cast<const double*>(v.data);
    a.out = static_cast<double*>(o.data);
    a.mirror = static_cast<double*>(mirror);
    a.q_b = q.str[0];
    a.q_t = q.str[1];
    a.q_h = q.str[2];
    a.o_b = o.str[0];
    a.o_t = o.str[1];
    a.o_h = o.str[2];
    a.o_d = o.str[3];
    a.o_pairs = o.str[3] == 1 && reinterpret_cast<uintptr_t>(o.data) % 16 == 0 && o.str[0] % 2 == 0 &&
                o.str[1] % 2 == 0 && o.str[2] % 2 == 0 && (mirror == nullptr || aligned(mirror, 16));
    a.k_b = k.str[0];
    a.k_h = k.str[head];
    a.k_t = k.str[tok];
    a.v_b = v.str[0];
    a.v_h = v.str[head];
    a.v_t = v.str[tok];
    a.Tq = q.ext[1];
    a.Tk = k.ext[tok];
    a.Hq = q.ext[2];
    a.g = g;
    a.causal = causal;
    int64_t const q_tiles = ceil_div(a.Tq, kBM), bhs = q.ext[0] * q.ext[2];
    if (q_tiles * bhs > INT32_MAX) return ANN_OK;  // not handled
    a.q_tiles = static_cast<int>(q_tiles);
    handled = true;
    if (D == 64) return launch_f64<64>(stream, a, scale, bhs);
    return launch_f64<128>(stream, a, scale, bhs);
}

int take_prefill_f64_error(cudaStream_t s, uint32_t* bits) {
    unsigned int value = 0, zero = 0;
    if (cudaMemcpyFromSymbolAsync(&value, g_f64_error, sizeof value, 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_f64_error, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ANN_ECUDA, "device error word: %s", cudaGetErrorString(cudaGetLastError()));
    *bits |= value;
    return ANN_OK;
}

}  // namespace ann
