// attention_ops.cu -- attentionScores / attentionApply as separate drop-in ops
// (reference: onHost/nn/attention.hpp:54-110, onAcc/internal/nn/attention.hpp:15-69).
//
// Both are batched contractions per (batch, query head):
//   scores: S[i,j] = sum_d Q[i,d] K[j,d]      (M=Tq, N=Tk, K=D)
//   apply:  O[i,d] = sum_j P[i,j] V[j,d]      (M=Tq, N=D,  K=Tk)
// with the KV head hq / queriesPerKvGroup (GQA) and K/V in BTHD or BHTD. One
// strided tiled kernel serves both: 64x64 output tiles, 16-deep K slices
// staged in shared memory with the global loads walking the unit-stride axis,
// 4x4 register blocking, FMA accumulation in ascending k per output -- the
// reference's summation order. These ops materialise the full score matrix
// like the reference does; the fused decode kernel is the fast path.
#include "common.cuh"

namespace ann {

// fp32 on the tensor cores (attention_tc.cu); `handled` = false when the
// shapes do not allow it and the FP32-pipe kernels below run instead
int scores_tc_f32(ann_stream stream, const Dims& q, const Dims& k, const Dims& s, uint32_t g, int layout,
                  bool& handled);
int apply_tc_f32(ann_stream stream, const Dims& p, const Dims& v, const Dims& o, uint32_t g, int layout,
                 bool& handled);

namespace {

struct BgemmArgs {
    const void* A;
    const void* B;
    void* C;
    int64_t M, N, K;
    int64_t am, ak, bk, bn, cm, cn;        // element strides inside one batch
    int64_t a_b, a_h, b_b, b_h, c_b, c_h;  // batch / head strides; B uses head hq / g
    int64_t heads;
    uint32_t g;
    int a_k_unit, b_k_unit;  // load mapping: walk k (1) or m/n (0) across threads
};

constexpr int BM = 64, BN = 64, BK = 16;

template <typename T>
__global__ void __launch_bounds__(256) bgemm_kernel(BgemmArgs a) {
    __shared__ T As[BK][BM + 1];
    __shared__ T Bs[BK][BN + 1];
    int const tid = threadIdx.x;
    int const tx = tid % 16, ty = tid / 16;
    int64_t const z = blockIdx.z;
    int64_t const b = z / a.heads, hq = z % a.heads;
    int64_t const kvh = hq / a.g;
    T const* A = static_cast<T const*>(a.A) + b * a.a_b + hq * a.a_h;
    T const* B = static_cast<T const*>(a.B) + b * a.b_b + kvh * a.b_h;
    T* C = static_cast<T*>(a.C) + b * a.c_b + hq * a.c_h;
    int64_t const m0 = static_cast<int64_t>(blockIdx.y) * BM, n0 = static_cast<int64_t>(blockIdx.x) * BN;
    T acc[4][4] = {};
    for (int64_t k0 = 0; k0 < a.K; k0 += BK) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int const lin = tid + e * 256;
            int const m = a.a_k_unit ? lin / BK : lin % BM;
            int const k = a.a_k_unit ? lin % BK : lin / BM;
            int64_t const gm = m0 + m, gk = k0 + k;
            As[k][m] = (gm < a.M && gk < a.K) ? A[gm * a.am + gk * a.ak] : T{};
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int const lin = tid + e * 256;
            int const n = a.b_k_unit ? lin / BK : lin % BN;
            int const k = a.b_k_unit ? lin % BK : lin / BN;
            int64_t const gn = n0 + n, gk = k0 + k;
            Bs[k][n] = (gn < a.N && gk < a.K) ? B[gk * a.bk + gn * a.bn] : T{};
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            T av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = As[k][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = Bs[k][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int64_t const gm = m0 + ty * 4 + i;
        if (gm >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int64_t const gn = n0 + tx * 4 + j;
            if (gn < a.N) C[gm * a.cm + gn * a.cn] = acc[i][j];
        }
    }
}

// fp32 at sizes that fill the GPU: 128-column x (16 TM)-row output tiles, 16-deep
// k slices (8-deep with scalar loads), each thread TM x 8 outputs in four quadrants (rows ty*TM/2 + i and
// BM/2 + ty*TM/2 + i, columns tx*4 + j and 64 + tx*4 + j) read from shared
// memory as 16-byte vectors. Two shared-memory buffers: the global loads of
// slice s + 1 go out before slice s is computed and land in the other buffer
// after it, one barrier per slice. Every output still accumulates k in
// ascending order with FMA, as bgemm_kernel does.
constexpr int BN128 = 128, PAD = 4;

// VL: both operands are loaded as 16-byte vectors (unit stride along the
// walked axis, 4-element aligned rows and extents), one or two a thread per
// slice, instead of TM + 4 scalar loads with their index arithmetic.
template <int TM, bool VL>
__global__ void __launch_bounds__(256, 2) bgemm_wide(BgemmArgs a, int vec_c) {
    constexpr int BMW = 16 * TM;
    constexpr int BK8 = VL ? 16 : 8;  // slice depth: 16 with 16-byte loads, 8 with scalar ones
    constexpr int LA = VL ? 1 : BMW * BK8 / 256, LB = VL ? 1 : BN128 * BK8 / 256;  // scalar loads a thread per slice
    constexpr int QA = BMW * BK8 / 4, QB = BN128 * BK8 / 4;  // 16-byte pieces of an A / B slice
    constexpr int VA = (QA + 255) / 256, VB = QB / 256;        // ... a thread (A: 2 or 1, B: 2)
    constexpr int PR = BK8 / 4;                                // pieces along k of one row
    __shared__ __align__(16) float As[2][BK8][BMW + PAD];
    __shared__ __align__(16) float Bs[2][BK8][BN128 + PAD];
    int const tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    int64_t const z = blockIdx.z;
    int64_t const b = z / a.heads, hq = z % a.heads;
    int64_t const kvh = hq / a.g;
    float const* A = static_cast<float const*>(a.A) + b * a.a_b + hq * a.a_h;
    float const* B = static_cast<float const*>(a.B) + b * a.b_b + kvh * a.b_h;
    float* C = static_cast<float*>(a.C) + b * a.c_b + hq * a.c_h;
    int64_t const m0 = static_cast<int64_t>(blockIdx.y) * BMW, n0 = static_cast<int64_t>(blockIdx.x) * BN128;
    float ra[LA], rb[LB];
    float4 va[VA], vb[VB];
    // piece q of a slice: along k, row q / PR at k (q % PR) * 4; along m / n,
    // k row q / (extent / 4) at (q % (extent / 4)) * 4
    auto load_vec = [&](int64_t k0) {
#pragma unroll
        for (int e = 0; e < VA; ++e) {
            int const q = tid + 256 * e;
            va[e] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (q < QA) {
                int64_t gm, gk;
                if (a.a_k_unit) gm = m0 + q / PR, gk = k0 + (q % PR) * 4;
                else gm = m0 + (q % (BMW / 4)) * 4, gk = k0 + q / (BMW / 4);
                if (gm < a.M && gk < a.K) va[e] = *reinterpret_cast<float4 const*>(A + gm * a.am + gk * a.ak);
            }
        }
#pragma unroll
        for (int e = 0; e < VB; ++e) {
            int const q = tid + 256 * e;
            int64_t gn, gk;
            if (a.b_k_unit) gn = n0 + q / PR, gk = k0 + (q % PR) * 4;
            else gn = n0 + (q % (BN128 / 4)) * 4, gk = k0 + q / (BN128 / 4);
            vb[e] = (gn < a.N && gk < a.K) ? *reinterpret_cast<float4 const*>(B + gk * a.bk + gn * a.bn)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store_vec = [&](int buf) {
#pragma unroll
        for (int e = 0; e < VA; ++e) {
            int const q = tid + 256 * e;
            if (q >= QA) continue;
            if (a.a_k_unit) {
                int const m = q / PR, k = (q % PR) * 4;
                As[buf][k][m] = va[e].x; As[buf][k + 1][m] = va[e].y; As[buf][k + 2][m] = va[e].z;
                As[buf][k + 3][m] = va[e].w;
            } else {
                *reinterpret_cast<float4*>(&As[buf][q / (BMW / 4)][(q % (BMW / 4)) * 4]) = va[e];
            }
        }
#pragma unroll
        for (int e = 0; e < VB; ++e) {
            int const q = tid + 256 * e;
            if (a.b_k_unit) {
                int const n = q / PR, k = (q % PR) * 4;
                Bs[buf][k][n] = vb[e].x; Bs[buf][k + 1][n] = vb[e].y; Bs[buf][k + 2][n] = vb[e].z;
                Bs[buf][k + 3][n] = vb[e].w;
            } else {
                *reinterpret_cast<float4*>(&Bs[buf][q / (BN128 / 4)][(q % (BN128 / 4)) * 4]) = vb[e];
            }
        }
    };
    auto load = [&](int64_t k0) {
        if constexpr (VL) {
            load_vec(k0);
        } else {
#pragma unroll
            for (int e = 0; e < LA; ++e) {
                int const lin = tid + e * 256;
                int const m = a.a_k_unit ? lin / BK8 : lin % BMW;
                int const k = a.a_k_unit ? lin % BK8 : lin / BMW;
                int64_t const gm = m0 + m, gk = k0 + k;
                ra[e] = (gm < a.M && gk < a.K) ? A[gm * a.am + gk * a.ak] : 0.f;
            }
#pragma unroll
            for (int e = 0; e < LB; ++e) {
                int const lin = tid + e * 256;
                int const n = a.b_k_unit ? lin / BK8 : lin % BN128;
                int const k = a.b_k_unit ? lin % BK8 : lin / BN128;
                int64_t const gn = n0 + n, gk = k0 + k;
                rb[e] = (gn < a.N && gk < a.K) ? B[gk * a.bk + gn * a.bn] : 0.f;
            }
        }
    };
    auto store = [&](int buf) {
        if constexpr (VL) {
            store_vec(buf);
        } else {
#pragma unroll
            for (int e = 0; e < LA; ++e) {
                int const lin = tid + e * 256;
                int const m = a.a_k_unit ? lin / BK8 : lin % BMW;
                int const k = a.a_k_unit ? lin % BK8 : lin / BMW;
                As[buf][k][m] = ra[e];
            }
#pragma unroll
            for (int e = 0; e < LB; ++e) {
                int const lin = tid + e * 256;
                int const n = a.b_k_unit ? lin / BK8 : lin % BN128;
                int const k = a.b_k_unit ? lin % BK8 : lin / BN128;
                Bs[buf][k][n] = rb[e];
            }
        }
    };
    float acc[TM][8];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    int64_t const slices = ceil_div(a.K, static_cast<int64_t>(BK8));
    load(0);
    store(0);
    __syncthreads();
    for (int64_t sl = 0; sl < slices; ++sl) {
        int const buf = static_cast<int>(sl & 1);
        if (sl + 1 < slices) load((sl + 1) * BK8);
#pragma unroll
        for (int k = 0; k < BK8; ++k) {
            float av[TM], bv[8];
            if constexpr (TM == 8) {  // 4 rows from each half: 16-byte aligned (ty * 4 floats)
                float4 const a0 = *reinterpret_cast<float4 const*>(&As[buf][k][ty * 4]);
                float4 const a1 = *reinterpret_cast<float4 const*>(&As[buf][k][BMW / 2 + ty * 4]);
                av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
                av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
            } else {  // TM == 4: 2 rows from each half, 8-byte aligned (ty * 2 floats)
                float2 const a0 = *reinterpret_cast<float2 const*>(&As[buf][k][ty * 2]);
                float2 const a1 = *reinterpret_cast<float2 const*>(&As[buf][k][BMW / 2 + ty * 2]);
                av[0] = a0.x; av[1] = a0.y; av[2] = a1.x; av[3] = a1.y;
            }
            float4 const b0 = *reinterpret_cast<float4 const*>(&Bs[buf][k][tx * 4]);
            float4 const b1 = *reinterpret_cast<float4 const*>(&Bs[buf][k][64 + tx * 4]);
            bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
            bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (sl + 1 < slices) store(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        int const half = i / (TM / 2), r = i % (TM / 2);
        int64_t const gm = m0 + half * (BMW / 2) + ty * (TM / 2) + r;
        if (gm >= a.M) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int64_t const gn = n0 + h * 64 + tx * 4;
            float* c = C + gm * a.cm;
            if (vec_c && gn + 3 < a.N) {
                *reinterpret_cast<float4*>(c + gn) =
                    make_float4(acc[i][4 * h], acc[i][4 * h + 1], acc[i][4 * h + 2], acc[i][4 * h + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (gn + j < a.N) c[(gn + j) * a.cn] = acc[i][4 * h + j];
            }
        }
    }
}

// fp64 on the FP64 tensor cores: mma.sync.m16n8k4.f64 (fp64 products and
// accumulation). 64 x 64 output tiles, 4 warps of 32 x 32 (2 x 4 MMA tiles of
// 16 x 8 each), 16-deep k slices in shared memory with k contiguous and a row
// pitch of 18 doubles (16 mod 128 bytes: each fragment read hits a bank at
// most twice per 256 bytes), two buffers, the next slice's global loads issued
// before the current one is computed. Fragments of m16n8k4.f64 (g = lane / 4,
// t = lane % 4): a0 = A[g][t], a1 = A[g + 8][t], b0 = B[t][g]; c0 = C[g][2t],
// c1 = C[g][2t + 1], c2 = C[g + 8][2t], c3 = C[g + 8][2t + 1].
constexpr int DM = 64, DN = 64, DK = 16, DP = DK + 2, kDThreads = 128;

__device__ __forceinline__ void dmma_acc(double (&c)[4], double a0, double a1, double b0) {
    asm volatile("mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
                 : "d"(a0), "d"(a1), "d"(b0));
}

__global__ void __launch_bounds__(kDThreads, 3) bgemm_dmma(BgemmArgs a) {
    constexpr int LA = DM * DK / kDThreads, LB = DN * DK / kDThreads;  // 8 loads each per slice
    __shared__ __align__(16) double As[2][DM][DP];
    __shared__ __align__(16) double Bs[2][DN][DP];
    int const tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int const g = lane >> 2, t = lane & 3;
    int const wm = warp >> 1, wn = warp & 1;
    int64_t const z = blockIdx.z;
    int64_t const b = z / a.heads, hq = z % a.heads;
    int64_t const kvh = hq / a.g;
    double const* A = static_cast<double const*>(a.A) + b * a.a_b + hq * a.a_h;
    double const* B = static_cast<double const*>(a.B) + b * a.b_b + kvh * a.b_h;
    double* C = static_cast<double*>(a.C) + b * a.c_b + hq * a.c_h;
    int64_t const m0 = static_cast<int64_t>(blockIdx.y) * DM, n0 = static_cast<int64_t>(blockIdx.x) * DN;
    double ra[LA], rb[LB];
    auto load = [&](int64_t k0) {
#pragma unroll
        for (int e = 0; e < LA; ++e) {
            int const lin = tid + e * kDThreads;
            int const m = a.a_k_unit ? lin / DK : lin % DM;
            int const k = a.a_k_unit ? lin % DK : lin / DM;
            int64_t const gm = m0 + m, gk = k0 + k;
            ra[e] = (gm < a.M && gk < a.K) ? A[gm * a.am + gk * a.ak] : 0.0;
        }
#pragma unroll
        for (int e = 0; e < LB; ++e) {
            int const lin = tid + e * kDThreads;
            int const n = a.b_k_unit ? lin / DK : lin % DN;
            int const k = a.b_k_unit ? lin % DK : lin / DN;
            int64_t const gn = n0 + n, gk = k0 + k;
            rb[e] = (gn < a.N && gk < a.K) ? B[gk * a.bk + gn * a.bn] : 0.0;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int e = 0; e < LA; ++e) {
            int const lin = tid + e * kDThreads;
            int const m = a.a_k_unit ? lin / DK : lin % DM;
            int const k = a.a_k_unit ? lin % DK : lin / DM;
            As[buf][m][k] = ra[e];
        }
#pragma unroll
        for (int e = 0; e < LB; ++e) {
            int const lin = tid + e * kDThreads;
            int const n = a.b_k_unit ? lin / DK : lin % DN;
            int const k = a.b_k_unit ? lin % DK : lin / DN;
            Bs[buf][n][k] = rb[e];
        }
    };
    double acc[2][4][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.0;
    int64_t const slices = ceil_div(a.K, static_cast<int64_t>(DK));
    load(0);
    store(0);
    __syncthreads();
    for (int64_t sl = 0; sl < slices; ++sl) {
        int const buf = static_cast<int>(sl & 1);
        if (sl + 1 < slices) load((sl + 1) * DK);
#pragma unroll
        for (int kk = 0; kk < DK / 4; ++kk) {
            double a0[2], a1[2], b0[4];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                a0[i] = As[buf][wm * 32 + 16 * i + g][4 * kk + t];
                a1[i] = As[buf][wm * 32 + 16 * i + g + 8][4 * kk + t];
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) b0[j] = Bs[buf][wn * 32 + 8 * j + g][4 * kk + t];
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) dmma_acc(acc[i][j], a0[i], a1[i], b0[j]);
        }
        if (sl + 1 < slices) store(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                int64_t const gm = m0 + wm * 32 + 16 * i + g + 8 * h;
                if (gm >= a.M) continue;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    int64_t const gn = n0 + wn * 32 + 8 * j + 2 * t + c;
                    if (gn < a.N) C[gm * a.cm + gn * a.cn] = acc[i][j][2 * h + c];
                }
            }
}

template <typename T>
int launch_bgemm(ann_stream stream, BgemmArgs& a, int64_t batches, const char* what) {
    a.a_k_unit = a.ak == 1 ? 1 : 0;
    a.b_k_unit = a.bk == 1 ? 1 : 0;
    if constexpr (sizeof(T) == 4) {
        // wide tiles once the problem fills the GPU; 64-row tiles when 128-row
        // ones would leave over a quarter of the CTA slots idle
        int64_t const gx = ceil_div(a.N, static_cast<int64_t>(BN128));
        int64_t const tiles128 = gx * ceil_div(a.M, int64_t{128}) * batches;
        int64_t const slots = static_cast<int64_t>(sm_count()) * 2;
        if (a.M >= 64 && a.N >= 64 && tiles128 >= slots / 2 && batches <= 65535) {
            int const vec_c = a.cn == 1 && a.cm % 4 == 0 && a.c_b % 4 == 0 && a.c_h % 4 == 0 && aligned(a.C, 16);
            bool const tall = 4 * tiles128 >= 3 * slots;
            int64_t const gy = ceil_div(a.M, tall ? int64_t{128} : int64_t{64});
            // 16-byte loads: along k (stride 1, row pitch and batch / head
            // strides multiples of 4, K a multiple of 4) or along m / n (the
            // same with M / N)
            auto vec_ok = [&](const void* base, int k_unit, int64_t s_k, int64_t s_o, int64_t sb, int64_t sh,
                              int64_t ext_o) {
                int64_t const unit = k_unit ? s_k : s_o, other = k_unit ? s_o : s_k;
                int64_t const walked = k_unit ? a.K : ext_o;
                return unit == 1 && other % 4 == 0 && sb % 4 == 0 && sh % 4 == 0 && walked % 4 == 0 &&
                       aligned(base, 16);
            };
            bool const vl = vec_ok(a.A, a.a_k_unit, a.ak, a.am, a.a_b, a.a_h, a.M) &&
                            vec_ok(a.B, a.b_k_unit, a.bk, a.bn, a.b_b, a.b_h, a.N);
            if (gy <= 65535) {
                dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy), static_cast<unsigned>(batches));
                cudaStream_t st = as_stream(stream);
                if (tall && vl) bgemm_wide<8, true><<<grid, 256, 0, st>>>(a, vec_c);
                else if (tall) bgemm_wide<8, false><<<grid, 256, 0, st>>>(a, vec_c);
                else if (vl) bgemm_wide<4, true><<<grid, 256, 0, st>>>(a, vec_c);
                else bgemm_wide<4, false><<<grid, 256, 0, st>>>(a, vec_c);
                return check_launch(what);
            }
        }
    }
    if constexpr (sizeof(T) == 8) {  // fp64: the FP64 tensor cores
        int64_t const gx = ceil_div(a.N, static_cast<int64_t>(DN)), gy = ceil_div(a.M, static_cast<int64_t>(DM));
        if (gy > 65535 || batches > 65535) return fail(ANN_ENOTSUP, "%s: grid too large for this build.", what);
        dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy), static_cast<unsigned>(batches));
        bgemm_dmma<<<grid, kDThreads, 0, as_stream(stream)>>>(a);
        return check_launch(what);
    }
    int64_t const gx = ceil_div(a.N, BN), gy = ceil_div(a.M, BM);
    if (gy > 65535 || batches > 65535) return fail(ANN_ENOTSUP, "%s: grid too large for this build.", what);
    dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy), static_cast<unsigned>(batches));
    bgemm_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(a);
    return check_launch(what);
}

int check_layout(int layout, const char* what) {
    if (layout != ANN_LAYOUT_BTHD && layout != ANN_LAYOUT_BHTD) return fail(ANN_EINVAL, "%s: invalid kv layout.", what);
    return ANN_OK;
}

template <typename T>
int attention_scores(ann_stream stream, const ann_view* q_v, const ann_view* k_v, const ann_view* s_v, uint32_t g,
                     int layout) {
    // attention.hpp:64-65
    if (g == 0u) return fail(ANN_EINVAL, "attentionScores requires queriesPerKvGroup > 0.");
    ANN_TRY(check_layout(layout, "attentionScores"));
    Dims q, k, s;
    ANN_TRY(to_dims(q_v, sizeof(T), "attentionScores Q", q));
    ANN_TRY(to_dims(k_v, sizeof(T), "attentionScores K", k));
    ANN_TRY(to_dims(s_v, sizeof(T), "attentionScores scores", s));
    if (q.rank != 4 || k.rank != 4 || s.rank != 4)
        return fail(ANN_EINVAL, "attentionScores expects rank-4 Q, K and scores.");
    int const tok = layout == ANN_LAYOUT_BTHD ? 1 : 2, head = layout == ANN_LAYOUT_BTHD ? 2 : 1;
    int64_t const B = s.ext[0], Hq = s.ext[1], Tq = s.ext[2], Tk = s.ext[3], D = q.ext[3];
    if (s.numel() == 0) return ANN_OK;
    // Reads the reference kernel would make out of bounds are rejected.
    if (q.ext[0] < B || q.ext[1] < Tq || q.ext[2] < Hq || k.ext[0] < B || k.ext[tok] < Tk ||
        k.ext[head] <= (Hq - 1) / static_cast<int64_t>(g) || k.ext[3] < D)
        return fail(ANN_EINVAL, "attentionScores: Q %s / K %s do not cover scores %s.", extents_str(q).c_str(),
                    extents_str(k).c_str(), extents_str(s).c_str());
    if constexpr (sizeof(T) == 4) {
        bool handled = false;
        int const rc = scores_tc_f32(stream, q, k, s, g, layout, handled);
        if (handled || rc != ANN_OK) return rc;
    }
    BgemmArgs a{};
    a.A = q.data;
    a.B = k.data;
    a.C = s.data;
    a.M = Tq;
    a.N = Tk;
    a.K = D;
    a.am = q.str[1];
    a.ak = q.str[3];
    a.bk = k.str[3];
    a.bn = k.str[tok];
    a.cm = s.str[2];
    a.cn = s.str[3];
    a.a_b = q.str[0];
    a.a_h = q.str[2];
    a.b_b = k.str[0];
    a.b_h = k.str[head];
    a.c_b = s.str[0];
    a.c_h = s.str[1];
    a.heads = Hq;
    a.g = g;
    return launch_bgemm<T>(stream, a, B * Hq, "attentionScores");
}

template <typename T>
int attention_apply(ann_stream stream, const ann_view* p_v, const ann_view* v_v, const ann_view* o_v, uint32_t g,
                    int layout) {
    // attention.hpp:93-94
    if (g == 0u) return fail(ANN_EINVAL, "attentionApply requires queriesPerKvGroup > 0.");
    ANN_TRY(check_layout(layout, "attentionApply"));
    Dims p, v, o;
    ANN_TRY(to_dims(p_v, sizeof(T), "attentionApply probs", p));
    ANN_TRY(to_dims(v_v, sizeof(T), "attentionApply values", v));
    ANN_TRY(to_dims(o_v, sizeof(T), "attentionApply out", o));
    if (p.rank != 4 || v.rank != 4 || o.rank != 4)
        return fail(ANN_EINVAL, "attentionApply expects rank-4 probs, values and out.");
    int const tok = layout == ANN_LAYOUT_BTHD ? 1 : 2, head = layout == ANN_LAYOUT_BTHD ? 2 : 1;
    int64_t const B = o.ext[0], Tq = o.ext[1], Hq = o.ext[2], D = o.ext[3], Tk = p.ext[3];
    if (o.numel() == 0) return ANN_OK;
    if (p.ext[0] < B || p.ext[1] < Hq || p.ext[2] < Tq || v.ext[0] < B || v.ext[tok] < Tk ||
        v.ext[head] <= (Hq - 1) / static_cast<int64_t>(g) || v.ext[3] < D)
        return fail(ANN_EINVAL, "attentionApply: probs %s / values %s do not cover out %s.", extents_str(p).c_str(),
                    extents_str(v).c_str(), extents_str(o).c_str());
    if constexpr (sizeof(T) == 4) {
        bool handled = false;
        int const rc = apply_tc_f32(stream, p, v, o, g, layout, handled);
        if (handled || rc != ANN_OK) return rc;
    }
    BgemmArgs a{};
    a.A = p.data;
    a.B = v.data;
    a.C = o.data;
    a.M = Tq;
    a.N = D;
    a.K = Tk;
    a.am = p.str[2];
    a.ak = p.str[3];
    a.bk = v.str[tok];
    a.bn = v.str[3];
    a.cm = o.str[1];
    a.cn = o.str[3];
    a.a_b = p.str[0];
    a.a_h = p.str[1];
    a.b_b = v.str[0];
    a.b_h = v.str[head];
    a.c_b = o.str[0];
    a.c_h = o.str[2];
    a.heads = Hq;
    a.g = g;
    return launch_bgemm<T>(stream, a, B * Hq, "attentionApply");
}

}  // namespace
}  // namespace ann

extern "C" {

int ann_attention_scores_f32(ann_stream s, const ann_view* q, const ann_view* k, const ann_view* sc, uint32_t g,
                             int32_t layout) {
    ANN_API_BEGIN
    return ann::attention_scores<float>(s, q, k, sc, g, layout);
    ANN_API_END
}
int ann_attention_scores_f64(ann_stream s, const ann_view* q, const ann_view* k, const ann_view* sc, uint32_t g,
                             int32_t layout) {
    ANN_API_BEGIN
    return ann::attention_scores<double>(s, q, k, sc, g, layout);
    ANN_API_END
}
int ann_attention_apply_f32(ann_stream s, const ann_view* p, const ann_view* v, const ann_view* o, uint32_t g,
                            int32_t layout) {
    ANN_API_BEGIN
    return ann::attention_apply<float>(s, p, v, o, g, layout);
    ANN_API_END
}
int ann_attention_apply_f64(ann_stream s, const ann_view* p, const ann_view* v, const ann_view* o, uint32_t g,
                            int32_t layout) {
    ANN_API_BEGIN
    return ann::attention_apply<double>(s, p, v, o, g, layout);
    ANN_API_END
}

}  // extern "C"
