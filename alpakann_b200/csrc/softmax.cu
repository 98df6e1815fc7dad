// softmax.cu -- softmax / causalSoftmax / maskedSoftmax (reference:
// onHost/nn/softmax.hpp:14-80, onAcc/internal/nn/softmax.hpp:15-116) and ops::scale
// (onHost/ops/elementwise.hpp:64-73, 330-334).
//
// Softmax rows run along an arbitrary axis of a tensor of any rank. A row of
// up to 8192 elements is owned by one to eight warps and held in their
// registers, 8, 16 or 32 elements per lane (one read, one write); a longer
// aligned row of up to 200 KB by a 256-thread CTA that brings it into shared
// memory with one bulk copy (one read, one write); an unaligned row of up to
// 96 KB by a CTA that loads it into shared memory itself; a longer row by a
// 256-thread CTA that re-reads it from L1/L2. In
// every case: max over the unmasked entries from lowest(), sum of
// exp(x - max), then out = exp(x - max) * (1 / sum) with masked entries
// written as 0 -- the reference's three passes, with the passes' reductions
// done by warp shuffles instead of one thread per row, and one division per
// row instead of one per element (the product is within an ulp of the
// reference's quotient; the per-element division made these kernels
// instruction-bound). The kept elements of a causal row are one index range,
// tested with one compare per element.
#include <type_traits>

#include <cooperative_groups.h>

#include "common.cuh"
#include "reduce.cuh"
#include "tma.cuh"

namespace ann {

int take_softmax_error(cudaStream_t s, uint32_t* bits);

namespace {

__device__ unsigned int g_softmax_error;  // ANN_DEVERR_WAIT_TIMEOUT from softmax_ring

struct SoftmaxArgs {
    const void* in;
    void* out;
    int64_t rows, len, s_in, s_out;  // row count, axis extent, axis strides
    Outer2 outer;                    // all axes, the softmax axis with extent 1
    int causal;
    int q_is_axis, k_is_axis;        // query / key axis coincides with the softmax axis
    int64_t q_div, q_mod, k_div, k_mod;  // component of the row index on the query / key axis
    const void* mask;                    // maskedSoftmax: additive mask, input's extents
    int64_t s_mask;                      // its stride along the softmax axis
    Outer2 mouter;                       // its row offsets (sa; sb unused)
    int uniform;                         // rows equally spaced in every operand:
    int64_t row_in, row_out, row_mask;   //   row r starts at r * row_* (no index division)
    int window;                          // softmax_ring copies only each row's kept window
};

// Row starts of row r in input, output and mask.
__device__ __forceinline__ void row_offsets(SoftmaxArgs const& a, int64_t row, int64_t& oi, int64_t& oo,
                                            int64_t& om) {
    if (a.uniform) {
        oi = row * a.row_in;
        oo = row * a.row_out;
        om = row * a.row_mask;
        return;
    }
    a.outer.offsets(row, oi, oo);
    int64_t unused;
    if (a.mask) a.mouter.offsets(row, om, unused);
}

// Elements of row `row` that the causal test keeps, as one range [lo, hi).
// An element e is kept when probe[queryAxis] >= probe[keyAxis] with
// probe[axis] = e, so with q, k the row's own query / key indices:
//   softmax axis = key axis only     e <= q   ->  [0, min(len, q + 1))
//   softmax axis = query axis only   e >= k   ->  [min(k, len), len)
//   softmax axis = both              always   ->  [0, len)
//   neither                          q >= k   ->  [0, len), else nothing.
// Without a causal mask every element is kept.
__device__ __forceinline__ void kept_range(SoftmaxArgs const& a, int64_t row, int64_t& lo, int64_t& hi) {
    lo = 0;
    hi = a.len;
    if (!a.causal) return;
    int64_t const q = (row / a.q_div) % a.q_mod, k = (row / a.k_div) % a.k_mod;
    if (a.k_is_axis && !a.q_is_axis) hi = q + 1 < a.len ? q + 1 : a.len;
    else if (a.q_is_axis && !a.k_is_axis) lo = k < a.len ? k : a.len;
    else if (!a.q_is_axis && !a.k_is_axis && q < k) hi = 0;
}

// A row of at most WPR * 32 * CH * VEC elements, owned by WPR warps and held
// in their registers: one read of the row, one write, nothing re-read. Lane
// l of warp w (of the row's WPR) owns the VEC-element pieces
// c * 32 * WPR + 32 w + l; with VEC > 1 (unit-stride, 16-byte aligned rows)
// each piece is one 16-byte load. All loads of a lane are issued before any
// of them is used. Max and sum: per lane in piece order, across the warp by
// shuffles, across the row's warps through shared memory in warp order.
template <typename T, int VEC>
struct Piece {
    using type = typename Vec16<T>::type;
};
template <typename T>
struct Piece<T, 1> {
    using type = T;
};

template <typename T, int CH, int VEC, int WPR, bool MASK>
__global__ void __launch_bounds__(256) softmax_regs(SoftmaxArgs a) {
    using P = typename Piece<T, VEC>::type;
    constexpr int N = CH * VEC;  // elements per lane
    constexpr int RPB = 8 / WPR;  // rows per CTA and iteration
    static_assert(N <= 64 && 8 % WPR == 0, "keep mask is 64 bits; WPR divides 8");
    // Partials of the row's warps, double-buffered by iteration parity, so
    // each reduction needs one barrier of the row's warps (named barrier
    // 1 + row group, 32 * WPR threads) and rows of a CTA never wait on each
    // other.
    __shared__ T red_max[2][8], red_sum[2][8];
    T const* in = static_cast<T const*>(a.in);
    T const* mk = static_cast<T const*>(a.mask);
    T* out = static_cast<T*>(a.out);
    int const lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int const part = warp % WPR, first = warp - part;  // this warp's slice; the row's first warp
    int64_t const per_iter = static_cast<int64_t>(gridDim.x) * RPB;
    int64_t const iters = ceil_div(a.rows, per_iter);
    for (int64_t it = 0; it < iters; ++it) {  // same trip count in every warp of the CTA
        int64_t const row = it * per_iter + static_cast<int64_t>(blockIdx.x) * RPB + warp / WPR;
        bool const live = row < a.rows;
        int64_t oi = 0, oo = 0, om = 0, lo64 = 0, hi64 = 0;
        if (live) {
            row_offsets(a, row, oi, oo, om);
            kept_range(a, row, lo64, hi64);
        }
        auto elem0 = [&](int c) { return (c * 32 * WPR + 32 * part + lane) * VEC; };  // < 8192 + 256
        T v[N];
        int const len = static_cast<int>(a.len);  // <= 8192 on this path
        // element e is kept iff lo <= e < hi: one unsigned compare
        int const lo = static_cast<int>(lo64);
        unsigned const span = hi64 > lo64 ? static_cast<unsigned>(hi64 - lo64) : 0u;
        auto kept = [&](int e) { return static_cast<unsigned>(e - lo) < span; };
        int const hi_k = lo + static_cast<int>(span);
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            int const e0 = elem0(c);
            // with VEC > 1, len is a multiple of VEC; pieces wholly outside the
            // kept range are not read (their values are never used)
            bool const in_row = live && e0 < len && e0 + VEC > lo && e0 < hi_k;
            P x{}, y{};
            if constexpr (VEC > 1) {
                if (in_row) x = *reinterpret_cast<P const*>(in + oi + e0);
                if constexpr (MASK)
                    if (in_row) y = *reinterpret_cast<P const*>(mk + om + e0);
            } else {
                if (in_row) x = in[oi + e0 * a.s_in];
                if constexpr (MASK)
                    if (in_row) y = mk[om + e0 * a.s_mask];
            }
            T const* xe = reinterpret_cast<T const*>(&x);
            T const* ye = reinterpret_cast<T const*>(&y);
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                if constexpr (MASK) v[c * VEC + k] = add_rn(xe[k], ye[k]);
                else v[c * VEC + k] = xe[k];
            }
        }
        // Elements outside [lo, hi), and slots past the row's end, become
        // -inf once, here: max ignores them and exp gives them exactly 0, so
        // the later passes need no tests. Rows with every slot kept skip it.
        bool const full = lo == 0 && span >= static_cast<unsigned>(32 * WPR * N);  // same in the whole row
        if (!full)
#pragma unroll
            for (int j = 0; j < N; ++j)
                if (!kept(elem0(j / VEC) + j % VEC)) v[j] = neg_inf(T{});
        T m = Lowest<T>::value;
#pragma unroll
        for (int j = 0; j < N; ++j) m = fmax(m, v[j]);
        int const buf = static_cast<int>(it & 1);
        auto row_barrier = [&]() {
            asm volatile("bar.sync %0, %1;" ::"r"(1 + warp / WPR), "r"(32 * WPR) : "memory");
        };
        m = warp_max(m);
        if constexpr (WPR > 1) {
            if (lane == 0) red_max[buf][warp] = m;
            row_barrier();
            m = red_max[buf][first];
#pragma unroll
            for (int w = 1; w < WPR; ++w) m = fmax(m, red_max[buf][first + w]);
        }
        // exp; in a row that is not fully kept, pieces wholly past the kept
        // range are 0 without evaluating exp (three quarters of a causal row
        // of 4096 against 1024 queries)
        int const hi = lo + static_cast<int>(span);
        T sum{};
        if (full) {
#pragma unroll
            for (int j = 0; j < N; ++j) {
                v[j] = exp_t(v[j] - m);
                sum += v[j];
            }
        } else {
#pragma unroll
            for (int j = 0; j < N; ++j) {
                v[j] = elem0(j / VEC) < hi ? exp_t(v[j] - m) : T(0);
                sum += v[j];
            }
        }
        sum = warp_sum(sum);
        if constexpr (WPR > 1) {
            if (lane == 0) red_sum[buf][warp] = sum;
            row_barrier();
            sum = red_sum[buf][first];
#pragma unroll
            for (int w = 1; w < WPR; ++w) sum += red_sum[buf][first + w];
        }
        if (!live) continue;
        // One division per row; x * (1 / sum) is within an ulp of x / sum.
        // sum >= 1 whenever a kept element is finite (the maximum contributes
        // exp(0)); otherwise (nothing kept, or only -inf / NaN kept) the
        // unkept slots are written as 0 explicitly, as the reference does.
        T const inv = T(1) / sum;
        auto store = [&](auto exact_tag) {
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                int const e0 = elem0(c);
                if (e0 >= len) continue;
                P r;
                T* re = reinterpret_cast<T*>(&r);
#pragma unroll
                for (int k = 0; k < VEC; ++k) {
                    if constexpr (decltype(exact_tag)::value) re[k] = kept(e0 + k) ? v[c * VEC + k] * inv : T{};
                    else re[k] = v[c * VEC + k] * inv;
                }
                if constexpr (VEC > 1) *reinterpret_cast<P*>(out + oo + e0) = r;
                else out[oo + e0 * a.s_out] = r;
            }
        };
        if (sum >= T(1)) store(std::false_type{});
        else store(std::true_type{});
    }
}

// Aligned rows of up to 8192 elements: softmax_regs' row groups and register
// layout, fed by a ring of bulk copies (TMA) instead of loads issued by the
// row's own threads. Warp 0 copies the input (and mask) rows of iteration
// it + STAGES - 1 into shared memory while the CTA computes iteration it, so a
// CTA keeps STAGES - 1 iterations of rows in flight whatever its threads are
// doing; the loads into registers then come from shared memory. Every wait is
// bounded: a copy that has not landed after 1 s sets ANN_DEVERR_WAIT_TIMEOUT,
// the CTA drains its copies in flight (bounded too) and returns.
template <typename T, int CH, int WPR, bool MASK>
struct RingCfg {
    static constexpr int NV = Vec16<T>::n;
    static constexpr int CAP = 32 * WPR * CH * NV;  // elements of one row slot
    static constexpr int RPB = 8 / WPR;              // rows a CTA takes per iteration
    static constexpr int OPS = MASK ? 2 : 1;         // input (+ mask) rows
    static constexpr int STAGE = RPB * CAP * OPS * static_cast<int>(sizeof(T));  // bytes
    static constexpr int STAGES = STAGE <= (8 << 10) ? 4 : STAGE <= (16 << 10) ? 3 : 2;
    static constexpr int SMEM = STAGE * STAGES;
};

template <typename T, int CH, int WPR, bool MASK>
__global__ void __launch_bounds__(256) softmax_ring(SoftmaxArgs a) {
    using C = RingCfg<T, CH, WPR, MASK>;
    using P = typename Vec16<T>::type;
    constexpr int NV = C::NV, N = CH * NV, RPB = C::RPB;
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ __align__(8) uint64_t full[C::STAGES];
    __shared__ T red_max[2][8], red_sum[2][8];
    T const* in = static_cast<T const*>(a.in);
    T const* mk = static_cast<T const*>(a.mask);
    T* out = static_cast<T*>(a.out);
    int const tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int const part = warp % WPR, first = warp - part, group = warp / WPR;
    int64_t const per_iter = static_cast<int64_t>(gridDim.x) * RPB;
    int64_t const iters = ceil_div(a.rows, per_iter);
    int const len = static_cast<int>(a.len);  // <= CAP, a multiple of NV
    uint32_t const row_bytes = static_cast<uint32_t>(len) * sizeof(T);
    uint32_t const bar0 = smem_u32(full), ring0 = smem_u32(ring);

    // Warp 0: the rows of iteration `it` into stage it % STAGES. One arrival
    // with the iteration's byte count, then one copy per row and operand.
    auto issue = [&](int64_t it) {
        int const st = static_cast<int>(it % C::STAGES);
        uint32_t const bar = bar0 + 8u * st;
        uint32_t const dst = ring0 + static_cast<uint32_t>(st) * C::STAGE;
        int64_t const r0 = it * per_iter + static_cast<int64_t>(blockIdx.x) * RPB;
        int64_t const left = a.rows - r0;  // the last iteration may hold fewer rows, or none
        int const live = static_cast<int>(left <= 0 ? 0 : left < RPB ? left : RPB);
        if (!a.window) {  // whole rows
            if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(live) * row_bytes * C::OPS);
            __syncwarp();
            if (lane < live) {
                int64_t oi, oo, om = 0;
                row_offsets(a, r0 + lane, oi, oo, om);
                bulk_copy_g2s(dst + static_cast<uint32_t>(lane * C::CAP * sizeof(T)), in + oi, row_bytes, bar);
                if constexpr (MASK)
                    bulk_copy_g2s(dst + static_cast<uint32_t>((RPB + lane) * C::CAP * sizeof(T)), mk + om, row_bytes,
                                  bar);
            }
            return;
        }
        // only the kept window of a causal row is copied (whole 16-byte pieces):
        // the reference never uses the values of masked elements
        int w0 = 0, w1 = 0;
        if (lane < live) {
            int64_t lo, hi;
            kept_range(a, r0 + lane, lo, hi);
            if (hi > lo) {
                w0 = static_cast<int>(lo) / NV * NV;
                w1 = static_cast<int>((hi + NV - 1) / NV * NV);
                if (w1 > len) w1 = len;
            }
        }
        uint32_t const bytes = static_cast<uint32_t>(w1 - w0) * sizeof(T);
        uint32_t const total = __reduce_add_sync(0xffffffffu, bytes);
        if (lane == 0) mbar_arrive_expect_tx(bar, total * C::OPS);
        __syncwarp();
        if (bytes > 0) {
            int64_t oi, oo, om = 0;
            row_offsets(a, r0 + lane, oi, oo, om);
            uint32_t const off = static_cast<uint32_t>(w0) * sizeof(T);
            bulk_copy_g2s(dst + static_cast<uint32_t>(lane * C::CAP * sizeof(T)) + off, in + oi + w0, bytes, bar);
            if constexpr (MASK)
                bulk_copy_g2s(dst + static_cast<uint32_t>((RPB + lane) * C::CAP * sizeof(T)) + off, mk + om + w0, bytes,
                              bar);
        }
    };

    if (tid == 0) {
        for (int st = 0; st < C::STAGES; ++st) mbar_init(bar0 + 8u * st, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == 0)
        for (int64_t it = 0; it < iters && it < C::STAGES; ++it) issue(it);

    auto row_barrier = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(1 + group), "r"(32 * WPR) : "memory"); };
    auto elem0 = [&](int c) { return (c * 32 * WPR + 32 * part + lane) * NV; };
    for (int64_t it = 0; it < iters; ++it) {
        int const st = static_cast<int>(it % C::STAGES);
        bool const ok = mbar_wait_bounded(bar0 + 8u * st, static_cast<uint32_t>((it / C::STAGES) & 1));
        // All threads agree on giving up; the barrier also retires every read
        // of the stage that iteration it - 1 used, which is refilled next.
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                atomicOr(&g_softmax_error, ANN_DEVERR_WAIT_TIMEOUT);
                for (int64_t u = it; u < iters && u < it - 1 + C::STAGES; ++u)  // copies in flight (bounded)
                    mbar_wait_bounded(bar0 + 8u * static_cast<uint32_t>(u % C::STAGES),
                                      static_cast<uint32_t>((u / C::STAGES) & 1));
            }
            return;
        }
        if (it >= 1 && warp == 0 && it - 1 + C::STAGES < iters) issue(it - 1 + C::STAGES);

        int64_t const row = it * per_iter + static_cast<int64_t>(blockIdx.x) * RPB + group;
        bool const live = row < a.rows;
        int64_t oi = 0, oo = 0, om = 0, lo64 = 0, hi64 = 0;
        if (live) {
            row_offsets(a, row, oi, oo, om);
            kept_range(a, row, lo64, hi64);
        }
        int const lo = static_cast<int>(lo64);
        unsigned const span = hi64 > lo64 ? static_cast<unsigned>(hi64 - lo64) : 0u;
        auto kept = [&](int e) { return static_cast<unsigned>(e - lo) < span; };
        T const* xs = reinterpret_cast<T const*>(ring + st * C::STAGE) + group * C::CAP;
        T const* ys = xs + RPB * C::CAP;
        T v[N];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            int const e0 = elem0(c);
            P x{}, y{};
            if (live && e0 < len) {
                x = *reinterpret_cast<P const*>(xs + e0);
                if constexpr (MASK) y = *reinterpret_cast<P const*>(ys + e0);
            }
            T const* xe = reinterpret_cast<T const*>(&x);
            T const* ye = reinterpret_cast<T const*>(&y);
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                if constexpr (MASK) v[c * NV + k] = add_rn(xe[k], ye[k]);
                else v[c * NV + k] = xe[k];
            }
        }
        bool const full = lo == 0 && span >= static_cast<unsigned>(C::CAP);  // as in softmax_regs
        if (!full)
#pragma unroll
            for (int j = 0; j < N; ++j)
                if (!kept(elem0(j / NV) + j % NV)) v[j] = neg_inf(T{});
        T m = Lowest<T>::value;
#pragma unroll
        for (int j = 0; j < N; ++j) m = fmax(m, v[j]);
        int const buf = static_cast<int>(it & 1);
        m = warp_max(m);
        if constexpr (WPR > 1) {
            if (lane == 0) red_max[buf][warp] = m;
            row_barrier();
            m = red_max[buf][first];
#pragma unroll
            for (int w = 1; w < WPR; ++w) m = fmax(m, red_max[buf][first + w]);
        }
        int const hi = lo + static_cast<int>(span);  // as in softmax_regs
        T sum{};
        if (full) {
#pragma unroll
            for (int j = 0; j < N; ++j) {
                v[j] = exp_t(v[j] - m);
                sum += v[j];
            }
        } else {
#pragma unroll
            for (int j = 0; j < N; ++j) {
                v[j] = elem0(j / NV) < hi ? exp_t(v[j] - m) : T(0);
                sum += v[j];
            }
        }
        sum = warp_sum(sum);
        if constexpr (WPR > 1) {
            if (lane == 0) red_sum[buf][warp] = sum;
            row_barrier();
            sum = red_sum[buf][first];
#pragma unroll
            for (int w = 1; w < WPR; ++w) sum += red_sum[buf][first + w];
        }
        if (!live) continue;
        T const inv = T(1) / sum;  // as in softmax_regs
        auto store = [&](auto exact_tag) {
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                int const e0 = elem0(c);
                if (e0 >= len) continue;
                P r;
                T* re = reinterpret_cast<T*>(&r);
#pragma unroll
                for (int k = 0; k < NV; ++k) {
                    if constexpr (decltype(exact_tag)::value) re[k] = kept(e0 + k) ? v[c * NV + k] * inv : T{};
                    else re[k] = v[c * NV + k] * inv;
                }
                *reinterpret_cast<P*>(out + oo + e0) = r;
            }
        };
        if (sum >= T(1)) store(std::false_type{});
        else store(std::true_type{});
    }
}

// Launches softmax_ring on a grid of resident CTAs (each streams its rows
// through its ring), or returns false when its ring does not fit a CTA.
template <typename T, int CH, int WPR, bool MASK>
bool launch_ring(SoftmaxArgs const& a, cudaStream_t s) {
    using C = RingCfg<T, CH, WPR, MASK>;
    if constexpr (C::SMEM > (200 << 10)) {
        return false;
    } else {
        auto kernel = softmax_ring<T, CH, WPR, MASK>;
        if (C::SMEM > (48 << 10) &&
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
            return false;
        static int per_sm = 0;  // same kernel, same B200 on every device of the process
        if (per_sm == 0 && (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, C::SMEM) != cudaSuccess ||
                            per_sm < 1)) {
            per_sm = 0;
            cudaGetLastError();
            return false;
        }
        int64_t const blocks = ceil_div(a.rows, static_cast<int64_t>(C::RPB));
        int64_t const cap = static_cast<int64_t>(sm_count()) * per_sm;
        kernel<<<static_cast<unsigned>(blocks < cap ? blocks : cap), 256, C::SMEM, s>>>(a);
        return true;
    }
}

// Rows longer than the register path holds but at most kSmemRowBytes: one
// 256-thread CTA per row, the row (input + mask for maskedSoftmax) kept in
// dynamic shared memory between the three passes, so it is read from HBM once
// and written once. Thread t owns the VEC-element pieces t, t + 256, ... in
// every pass, so no thread reads an element another one wrote and the only
// barriers are the two inside the block reductions. Loads go out kBatch
// pieces at a time before any of them is used.
constexpr int64_t kSmemRowBytes = int64_t{96} << 10;
constexpr int kBatch = 4;

template <typename T, int VEC, bool MASK>
__global__ void __launch_bounds__(256) softmax_smem(SoftmaxArgs a) {
    using P = typename Piece<T, VEC>::type;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* buf = reinterpret_cast<T*>(smem_raw);
    __shared__ T scratch[8];
    T const* in = static_cast<T const*>(a.in);
    T const* mk = static_cast<T const*>(a.mask);
    T* out = static_cast<T*>(a.out);
    int64_t const pieces = a.len / VEC;  // with VEC > 1, len is a multiple of VEC
    for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {  // same trip count in the whole CTA
        int64_t oi = 0, oo = 0, om = 0, lo = 0, hi = 0;
        row_offsets(a, row, oi, oo, om);
        kept_range(a, row, lo, hi);
        auto masked = [&](int64_t e) { return e < lo || e >= hi; };
        T m = Lowest<T>::value;
        for (int64_t p0 = threadIdx.x; p0 < pieces; p0 += 256 * kBatch) {
            P x[kBatch], y[kBatch];
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                int64_t const e0 = (p0 + 256 * u) * VEC;
                x[u] = P{};
                y[u] = P{};
                if (p0 + 256 * u >= pieces) continue;
                if (e0 + VEC <= lo || e0 >= hi) continue;  // wholly masked: its values are never used
                if constexpr (VEC > 1) {
                    x[u] = *reinterpret_cast<P const*>(in + oi + e0);
                    if constexpr (MASK) y[u] = *reinterpret_cast<P const*>(mk + om + e0);
                } else {
                    x[u] = in[oi + e0 * a.s_in];
                    if constexpr (MASK) y[u] = mk[om + e0 * a.s_mask];
                }
            }
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                int64_t const e0 = (p0 + 256 * u) * VEC;
                if (p0 + 256 * u >= pieces) continue;
                T* xe = reinterpret_cast<T*>(&x[u]);
                T const* ye = reinterpret_cast<T const*>(&y[u]);
#pragma unroll
                for (int k = 0; k < VEC; ++k) {
                    if constexpr (MASK) xe[k] = add_rn(xe[k], ye[k]);
                    if (masked(e0 + k)) xe[k] = neg_inf(T{});  // exp of it is exactly 0 below
                    m = fmax(m, xe[k]);
                }
                *reinterpret_cast<P*>(buf + e0) = x[u];
            }
        }
        m = block_max<8>(m, scratch);
        T sum{};
        for (int64_t p = threadIdx.x; p < pieces; p += 256) {
            int64_t const e0 = p * VEC;
            P x = *reinterpret_cast<P const*>(buf + e0);
            T* xe = reinterpret_cast<T*>(&x);
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                xe[k] = exp_t(xe[k] - m);
                sum += xe[k];
            }
            *reinterpret_cast<P*>(buf + e0) = x;
        }
        sum = block_sum<8>(sum, scratch);
        // one division per row; x * (1 / sum) is within an ulp of x / sum;
        // unkept slots tested only when sum < 1 (see softmax_regs)
        T const inv = T(1) / sum;
        bool const exact = !(sum >= T(1));
        for (int64_t p = threadIdx.x; p < pieces; p += 256) {
            int64_t const e0 = p * VEC;
            P x = *reinterpret_cast<P const*>(buf + e0);
            T* xe = reinterpret_cast<T*>(&x);
#pragma unroll
            for (int k = 0; k < VEC; ++k) xe[k] = exact && masked(e0 + k) ? T(0) : xe[k] * inv;
            if constexpr (VEC > 1) *reinterpret_cast<P*>(out + oo + e0) = x;
            else out[oo + e0 * a.s_out] = x;
        }
    }
}

// Aligned rows longer than the register path holds, up to kBulkBytes of
// input (+ mask): one CTA per row, the whole row brought into shared memory by
// ONE bulk copy (TMA) -- all of it in flight at once, where per-thread loads
// keep a few pieces a thread in flight -- and, with two stages, the next
// row's copy issued while this one is computed. Then softmax_smem's passes
// over shared memory (masked slots -inf from the first pass on, one
// reciprocal a row). Every wait is bounded: a copy that has not landed after
// 1 s sets ANN_DEVERR_WAIT_TIMEOUT, the CTA drains its copies in flight
// (bounded too) and returns.
constexpr int64_t kBulkBytes = int64_t{200} << 10;

template <typename T, bool MASK>
__global__ void __launch_bounds__(256) softmax_bulk(SoftmaxArgs a, int stages, uint32_t stage_bytes) {
    using P = typename Vec16<T>::type;
    constexpr int NV = Vec16<T>::n;
    extern __shared__ __align__(128) unsigned char rows_smem[];
    __shared__ __align__(8) uint64_t full[2];
    __shared__ T scratch[8];
    T const* in = static_cast<T const*>(a.in);
    T const* mk = static_cast<T const*>(a.mask);
    T* out = static_cast<T*>(a.out);
    int const tid = threadIdx.x;
    int64_t const pieces = a.len / NV;
    uint32_t const row_bytes = static_cast<uint32_t>(a.len) * sizeof(T);
    int64_t const iters = ceil_div(a.rows - static_cast<int64_t>(blockIdx.x), static_cast<int64_t>(gridDim.x));
    uint32_t const bar0 = smem_u32(full), base0 = smem_u32(rows_smem);
    auto issue = [&](int64_t it) {  // thread 0: row blockIdx.x + it * gridDim.x into stage it % stages
        int const st = static_cast<int>(it % stages);
        int64_t const row = static_cast<int64_t>(blockIdx.x) + it * gridDim.x;
        int64_t oi, oo, om = 0;
        row_offsets(a, row, oi, oo, om);
        uint32_t const bar = bar0 + 8u * st, dst = base0 + static_cast<uint32_t>(st) * stage_bytes;
        // only the kept window of a causal row is copied (whole 16-byte pieces)
        int64_t lo, hi, w0 = 0, w1 = 0;
        kept_range(a, row, lo, hi);
        if (hi > lo) {
            w0 = lo / NV * NV;
            w1 = (hi + NV - 1) / NV * NV;
            if (w1 > a.len) w1 = a.len;
        }
        uint32_t const bytes = static_cast<uint32_t>(w1 - w0) * sizeof(T);
        mbar_arrive_expect_tx(bar, bytes + (MASK ? row_bytes : 0u));
        if (bytes > 0) bulk_copy_g2s(dst + static_cast<uint32_t>(w0) * sizeof(T), in + oi + w0, bytes, bar);
        if constexpr (MASK) bulk_copy_g2s(dst + row_bytes, mk + om, row_bytes, bar);
    };
    if (tid == 0) {
        for (int st = 0; st < stages; ++st) mbar_init(bar0 + 8u * st, 1);
        fence_mbar_init();
        for (int64_t it = 0; it < iters && it < stages; ++it) issue(it);
    }
    __syncthreads();
    for (int64_t it = 0; it < iters; ++it) {
        int const st = static_cast<int>(it % stages);
        bool const ok = mbar_wait_bounded(bar0 + 8u * st, static_cast<uint32_t>((it / stages) & 1));
        if (__syncthreads_or(!ok)) {  // all threads agree on giving up
            if (tid == 0) {
                atomicOr(&g_softmax_error, ANN_DEVERR_WAIT_TIMEOUT);
                for (int64_t u = it; u < iters && u < it + stages; ++u)  // copies in flight (bounded)
                    mbar_wait_bounded(bar0 + 8u * static_cast<uint32_t>(u % stages),
                                      static_cast<uint32_t>((u / stages) & 1));
            }
            return;
        }
        int64_t const row = static_cast<int64_t>(blockIdx.x) + it * gridDim.x;
        int64_t oi, oo, om = 0, lo, hi;
        row_offsets(a, row, oi, oo, om);
        kept_range(a, row, lo, hi);
        T* buf = reinterpret_cast<T*>(rows_smem + static_cast<size_t>(st) * stage_bytes);
        T const* mbuf = buf + a.len;
        T m = Lowest<T>::value;
        for (int64_t p = tid; p < pieces; p += 256) {
            int64_t const e0 = p * NV;
            P x = *reinterpret_cast<P const*>(buf + e0);
            T* xe = reinterpret_cast<T*>(&x);
            if constexpr (MASK) {
                P const y = *reinterpret_cast<P const*>(mbuf + e0);
                T const* ye = reinterpret_cast<T const*>(&y);
#pragma unroll
                for (int k = 0; k < NV; ++k) xe[k] = add_rn(xe[k], ye[k]);
            }
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                if (e0 + k < lo || e0 + k >= hi) xe[k] = neg_inf(T{});  // exp of it is exactly 0 below
                m = fmax(m, xe[k]);
            }
            *reinterpret_cast<P*>(buf + e0) = x;
        }
        m = block_max<8>(m, scratch);
        T sum{};
        for (int64_t p = tid; p < pieces; p += 256) {
            int64_t const e0 = p * NV;
            P x = *reinterpret_cast<P const*>(buf + e0);
            T* xe = reinterpret_cast<T*>(&x);
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                xe[k] = exp_t(xe[k] - m);
                sum += xe[k];
            }
            *reinterpret_cast<P*>(buf + e0) = x;
        }
        sum = block_sum<8>(sum, scratch);
        // one division per row; unkept slots tested only when sum < 1 (see softmax_regs)
        T const inv = T(1) / sum;
        bool const exact = !(sum >= T(1));
        for (int64_t p = tid; p < pieces; p += 256) {
            int64_t const e0 = p * NV;
            P x = *reinterpret_cast<P const*>(buf + e0);
            T* xe = reinterpret_cast<T*>(&x);
#pragma unroll
            for (int k = 0; k < NV; ++k) xe[k] = exact && (e0 + k < lo || e0 + k >= hi) ? T(0) : xe[k] * inv;
            *reinterpret_cast<P*>(out + oo + e0) = x;
        }
        // every read of stage st is done: refill it with the row `stages`
        // iterations on (issued here, not at the next iteration's start, so
        // that one stage works too)
        __syncthreads();
        if (tid == 0 && it + stages < iters) issue(it + stages);
    }
}

// Launches softmax_bulk on a grid of resident CTAs; false when one row does
// not fit. One row stage a CTA: several CTAs an SM, each with a whole row in
// flight, kept more bytes in flight than two stages in fewer CTAs (rows of
// 16384 fp32: 0.85 of the copy peak against 0.67).
template <typename T, bool MASK>
bool bulk_launched(SoftmaxArgs const& a, cudaStream_t s) {
    int64_t const stage = ceil_div(a.len * static_cast<int64_t>(sizeof(T)) * (MASK ? 2 : 1), int64_t{128}) * 128;
    if (stage > kBulkBytes) return false;
    int const stages = 1;
    int const smem = static_cast<int>(stage * stages);
    auto kernel = softmax_bulk<T, MASK>;
    if (smem > (48 << 10) &&
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, smem) != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        return false;
    }
    int64_t const cap = static_cast<int64_t>(sm_count()) * per_sm;
    kernel<<<static_cast<unsigned>(a.rows < cap ? a.rows : cap), 256, smem, s>>>(a, stages,
                                                                              static_cast<uint32_t>(stage));
    return true;
}

// Long aligned rows (over 64 KB of input + mask) split over a cluster of
// kSplit CTAs. CTA s brings the s-th part of the row into its shared memory by
// one bulk copy and reads it into registers (at most kSplitVecs 16-byte pieces
// a thread), and at once issues the copy of its part of the next row into the
// same buffer: a copy is in flight while the row is reduced, exponentiated and
// written, and the buffer stays one stage (several clusters an SM). Max and
// sum: the CTA reduces its part (shuffles, then one warp over the per-warp
// values), and one lane per peer sends the CTA's value into that peer's
// exchange slot with st.async, completing on the peer's mbarrier; every CTA
// combines the kSplit values in rank order, so all hold the same max and sum.
// No cluster-wide barrier inside the row loop: its release would wait for
// this CTA's output stores of the previous row to drain. Waits are bounded; a
// CTA whose copy does not land sets ANN_DEVERR_WAIT_TIMEOUT and keeps sending
// its (empty) values without issuing more copies; an exchange that does not
// complete sets the same bit and the CTA stops waiting on exchanges.
constexpr int kSplit = 4, kSplitVecs = 8;
constexpr int64_t kSplitMinBytes = int64_t{64} << 10, kSplitPartBytes = int64_t{56} << 10;

template <typename T, bool MASK, int THREADS, int MINB>
__global__ void __launch_bounds__(THREADS, MINB) softmax_cluster(SoftmaxArgs a) {
    namespace cg = cooperative_groups;
    using P = typename Vec16<T>::type;
    constexpr int NV = Vec16<T>::n, WARPS = THREADS / 32;
    static_assert(WARPS <= 32 && kSplit <= 32, "one warp combines the warps' values and sends to the peers");
    extern __shared__ __align__(128) unsigned char part_smem[];
    __shared__ __align__(8) uint64_t full;
    __shared__ __align__(8) uint64_t xbar[2][2];  // [row parity][max, sum]: the peers' values have arrived
    __shared__ T xv[2][2][kSplit];                // [row parity][max, sum][source CTA]
    __shared__ T red[2][WARPS];                   // per-warp max / sum of this CTA
    int const tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int const s = static_cast<int>(cluster_ctarank());
    int64_t const part = a.len / kSplit, e_begin = s * part;
    int const np = static_cast<int>(part / NV);  // pieces of this CTA's part, <= kSplitVecs * THREADS
    uint32_t const part_bytes = static_cast<uint32_t>(part) * sizeof(T);
    int64_t const n_clusters = gridDim.x / kSplit, cid = blockIdx.x / kSplit;
    int64_t const iters = ceil_div(a.rows - cid, n_clusters);
    uint32_t const bar = smem_u32(&full), dst = smem_u32(part_smem);
    T const* in = static_cast<T const*>(a.in);
    T const* mk = static_cast<T const*>(a.mask);
    T* out = static_cast<T*>(a.out);
    T const* buf = reinterpret_cast<T const*>(part_smem);
    T const* mbuf = buf + part;
    auto issue = [&](int64_t it) {  // thread 0: this CTA's part of row cid + it * n_clusters
        int64_t oi, oo, om = 0, lo, hi;
        row_offsets(a, cid + it * n_clusters, oi, oo, om);
        // only the kept window of a causal row within this part is copied
        kept_range(a, cid + it * n_clusters, lo, hi);
        int64_t w0 = e_begin, w1 = e_begin + part;
        if (hi <= lo) {
            w1 = w0;
        } else {
            if (lo / NV * NV > w0) w0 = lo / NV * NV;
            if ((hi + NV - 1) / NV * NV < w1) w1 = (hi + NV - 1) / NV * NV;
            if (w1 < w0) w1 = w0;
        }
        uint32_t const bytes = static_cast<uint32_t>(w1 - w0) * sizeof(T);
        mbar_arrive_expect_tx(bar, bytes + (MASK ? part_bytes : 0u));
        if (bytes > 0) bulk_copy_g2s(dst + static_cast<uint32_t>(w0 - e_begin) * sizeof(T), in + oi + w0, bytes, bar);
        if constexpr (MASK) bulk_copy_g2s(dst + part_bytes, mk + om + e_begin, part_bytes, bar);
    };
    if (tid == 0) {
        mbar_init(bar, 1);
        for (int p = 0; p < 2; ++p)
            for (int k = 0; k < 2; ++k) mbar_init(smem_u32(&xbar[p][k]), 1);
        fence_mbar_init();
        if (iters > 0) issue(0);
    }
    __syncthreads();
    cg::this_cluster().sync();  // every peer's exchange barriers exist before the first value is sent to them
    bool dead = false;          // a copy did not land: no more copies, but every exchange is still joined
    bool lost = false;          // an exchange did not complete: no more waits on exchanges
    // The row's max (K = 0) or sum (K = 1) over the cluster, from this thread's
    // partial v; `at_barrier` runs in thread 0 once every thread has arrived.
    auto exchange = [&](T v, int K, int64_t it, auto&& at_barrier) -> T {
        v = K == 0 ? warp_max(v) : warp_sum(v);
        if (lane == 0) red[K][warp] = v;
        __syncthreads();
        if (tid == 0) at_barrier();
        int const par = static_cast<int>(it & 1);
        uint32_t const xb = smem_u32(&xbar[par][K]);
        if (warp == 0) {
            T c = lane < WARPS ? red[K][lane] : (K == 0 ? Lowest<T>::value : T(0));
            c = K == 0 ? warp_max(c) : warp_sum(c);
            if (lane == 0) mbar_arrive_expect_tx(xb, kSplit * sizeof(T));
            if (lane < kSplit) st_async_cluster(map_cluster(smem_u32(&xv[par][K][s]), lane), c, map_cluster(xb, lane));
        }
        if (!lost && !mbar_wait_bounded<true>(xb, static_cast<uint32_t>((it >> 1) & 1))) {
            if (tid == 0) atomicOr(&g_softmax_error, ANN_DEVERR_WAIT_TIMEOUT);
            lost = true;
        }
        T r = xv[par][K][0];
#pragma unroll
        for (int q = 1; q < kSplit; ++q) r = K == 0 ? fmax(r, xv[par][K][q]) : r + xv[par][K][q];
        return r;
    };
    for (int64_t it = 0; it < iters; ++it) {
        int64_t const row = cid + it * n_clusters;
        int64_t oi, oo, om = 0, lo, hi;
        row_offsets(a, row, oi, oo, om);
        kept_range(a, row, lo, hi);
        bool const ok = dead || mbar_wait_bounded(bar, static_cast<uint32_t>(it & 1));
        if (__syncthreads_or(!ok)) {
            if (tid == 0 && !dead) {
                atomicOr(&g_softmax_error, ANN_DEVERR_WAIT_TIMEOUT);
                mbar_wait_bounded(bar, static_cast<uint32_t>(it & 1));  // the copy in flight (bounded)
            }
            dead = true;
        }
        // the kept range [lo, hi) within this CTA's part, in 32-bit; a part kept
        // whole (every non-causal row) takes the loops without per-element tests
        int const plo = static_cast<int>(lo - e_begin < 0 ? 0 : (lo - e_begin > part ? part : lo - e_begin));
        int const phi = static_cast<int>(hi - e_begin < 0 ? 0 : (hi - e_begin > part ? part : hi - e_begin));
        bool const whole = plo == 0 && phi == static_cast<int>(part);
        P v[kSplitVecs];
        T m = Lowest<T>::value;
        if (!dead) {
#pragma unroll
            for (int j = 0; j < kSplitVecs; ++j) {
                int const p = tid + j * THREADS;
                if (p >= np) break;
                int const e0 = p * NV;
                v[j] = *reinterpret_cast<P const*>(buf + e0);
                T* xe = reinterpret_cast<T*>(&v[j]);
                if constexpr (MASK) {
                    P const y = *reinterpret_cast<P const*>(mbuf + e0);
                    T const* ye = reinterpret_cast<T const*>(&y);
#pragma unroll
                    for (int k = 0; k < NV; ++k) xe[k] = add_rn(xe[k], ye[k]);
                }
                if (whole) {
#pragma unroll
                    for (int k = 0; k < NV; ++k) m = fmax(m, xe[k]);
                } else {
#pragma unroll
                    for (int k = 0; k < NV; ++k) {
                        if (e0 + k < plo || e0 + k >= phi) xe[k] = neg_inf(T{});  // exp of it is exactly 0 below
                        m = fmax(m, xe[k]);
                    }
                }
            }
        }
        // every thread holds its pieces once it reaches the exchange's CTA
        // barrier: the buffer takes the next row's part from there on
        T const M = exchange(m, 0, it, [&] {
            if (!dead && it + 1 < iters) issue(it + 1);
        });
        T sum{};
        if (!dead) {
#pragma unroll
            for (int j = 0; j < kSplitVecs; ++j) {
                if (tid + j * THREADS >= np) break;
                T* xe = reinterpret_cast<T*>(&v[j]);
#pragma unroll
                for (int k = 0; k < NV; ++k) {
                    xe[k] = exp_t(xe[k] - M);
                    sum += xe[k];
                }
            }
        }
        T const L = exchange(sum, 1, it, [] {});
        // one division per row; unkept slots tested only when the sum < 1 (see softmax_regs)
        T const inv = T(1) / L;
        bool const exact = !(L >= T(1));
        if (!dead) {
            bool const plain = whole || !exact;
            T* orow = out + oo + e_begin;
#pragma unroll
            for (int j = 0; j < kSplitVecs; ++j) {
                int const p = tid + j * THREADS;
                if (p >= np) break;
                int const e0 = p * NV;
                T* xe = reinterpret_cast<T*>(&v[j]);
                if (plain) {
#pragma unroll
                    for (int k = 0; k < NV; ++k) xe[k] = xe[k] * inv;
                } else {
#pragma unroll
                    for (int k = 0; k < NV; ++k) xe[k] = (e0 + k < plo || e0 + k >= phi) ? T(0) : xe[k] * inv;
                }
                *reinterpret_cast<P*>(orow + e0) = v[j];
            }
        }
    }
    cg::this_cluster().sync();  // no CTA leaves while a peer's value may still be on its way to it
}

// Launches softmax_cluster<T, MASK, THREADS, MINB> on a grid of resident
// clusters. MINB caps the registers: fp32 rows of 32768 on B200 (back-to-back
// launches) took 90.6 us with three CTAs of 80 registers an SM = 0.90 of the
// measured copy rate; two CTAs of 128 registers, or four of 64 with spills,
// were slower (single launches: 115 and 132 us against 104). Two copy stages
// a CTA (93.3 us) and clusters of eight CTAs (92.7) did not pay either.
template <typename T, bool MASK, int THREADS, int MINB>
bool cluster_launch(SoftmaxArgs const& a, int smem, cudaStream_t s) {
    auto kernel = softmax_cluster<T, MASK, THREADS, MINB>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute cl{};
    cl.id = cudaLaunchAttributeClusterDimension;
    cl.val.clusterDim.x = kSplit;
    cl.val.clusterDim.y = 1;
    cl.val.clusterDim.z = 1;
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = s;
    cfg.attrs = &cl;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(kSplit);
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess || clusters < 1) {
        cudaGetLastError();
        return false;
    }
    int64_t const n = a.rows < clusters ? a.rows : clusters;
    cfg.gridDim = dim3(static_cast<unsigned>(n * kSplit));
    return cudaLaunchKernelEx(&cfg, kernel, a) == cudaSuccess;
}

// softmax_cluster where it applies: 256 threads a CTA while a part fits their
// registers (kSplitVecs pieces a thread: rows up to 32768 fp32 / 16384 fp64),
// 512 beyond; false when it does not apply.
template <typename T, bool MASK>
bool cluster_launched(SoftmaxArgs const& a, cudaStream_t s) {
    int64_t const bytes = a.len * static_cast<int64_t>(sizeof(T)) * (MASK ? 2 : 1);
    constexpr int NV = Vec16<T>::n;
    if (bytes <= kSplitMinBytes || bytes > kSplit * kSplitPartBytes || a.len % (kSplit * NV) != 0) return false;
    int const smem = static_cast<int>(bytes / kSplit);
    int64_t const pieces = a.len / kSplit / NV;
    constexpr bool f32 = sizeof(T) == 4;  // fp64 exp needs more registers: one CTA fewer an SM
    if (pieces <= int64_t{kSplitVecs} * 256) return cluster_launch<T, MASK, 256, f32 ? 3 : 2>(a, smem, s);
    if (pieces <= int64_t{kSplitVecs} * 512) return cluster_launch<T, MASK, 512, f32 ? 2 : 1>(a, smem, s);
    return false;
}

// MASK: maskedSoftmax (onAcc/internal/nn/softmax.hpp:76-116), the row is
// input + mask and nothing is skipped.
template <typename T, int GROUP, bool MASK>
__global__ void __launch_bounds__(256) softmax_kernel(SoftmaxArgs a) {
    constexpr int RPB = 256 / GROUP;
    __shared__ T scratch[8];
    int const gl = threadIdx.x % GROUP;
    T const* in = static_cast<T const*>(a.in);
    T* out = static_cast<T*>(a.out);
    int64_t const iters = ceil_div(a.rows, static_cast<int64_t>(gridDim.x) * RPB);
    for (int64_t it = 0; it < iters; ++it) {
        int64_t const row = (it * gridDim.x + blockIdx.x) * RPB + threadIdx.x / GROUP;
        bool const live = row < a.rows;
        int64_t oi = 0, oo = 0, om = 0, lo = 0, hi = 0;
        if (live) {
            row_offsets(a, row, oi, oo, om);
            kept_range(a, row, lo, hi);
        }
        auto masked = [&](int64_t i) { return i < lo || i >= hi; };
        T const* mk = static_cast<T const*>(a.mask);
        auto value = [&](int64_t i) {
            if constexpr (MASK) return add_rn(in[oi + i * a.s_in], mk[om + i * a.s_mask]);
            else return in[oi + i * a.s_in];
        };
        T m = Lowest<T>::value;
        if (live)
            for (int64_t i = gl; i < a.len; i += GROUP)
                if (!masked(i)) m = fmax(m, value(i));
        if constexpr (GROUP == 32) m = warp_max(m);
        else m = block_max<8>(m, scratch);
        T sum{};
        if (live)
            for (int64_t i = gl; i < a.len; i += GROUP)
                if (!masked(i)) sum += exp_t(value(i) - m);
        if constexpr (GROUP == 32) sum = warp_sum(sum);
        else sum = block_sum<8>(sum, scratch);
        if (!live) continue;
        T const inv = T(1) / sum;  // one division per row; x * (1 / sum) is within an ulp of x / sum
        for (int64_t i = gl; i < a.len; i += GROUP) {
            T const v = masked(i) ? T{} : exp_t(value(i) - m) * inv;
            out[oo + i * a.s_out] = v;
        }
    }
}

// softmax_ring for an aligned row of at most 8192 elements: the tier of
// softmax_regs that the row length picks (CV 16-byte pieces a lane at up to
// 2048 elements).
template <typename T, int CV, bool M>
bool ring_launched(SoftmaxArgs const& a, cudaStream_t s) {
    if (a.len <= 256) return launch_ring<T, CV, 1, M>(a, s);
    if (a.len <= 512) return launch_ring<T, CV, 2, M>(a, s);
    if (a.len <= 1024) return launch_ring<T, CV, 4, M>(a, s);
    if (a.len <= 2048) return launch_ring<T, CV, 8, M>(a, s);
    if (a.len <= 4096) return launch_ring<T, 2 * CV, 8, M>(a, s);
    return launch_ring<T, 4 * CV, 8, M>(a, s);
}

template <typename T>
int softmax(ann_stream stream, const ann_view* in_v, const ann_view* out_v, uint32_t axis, bool causal,
            uint32_t qaxis, uint32_t kaxis, const ann_view* mask_v = nullptr) {
    Dims in, out, mask;
    ANN_TRY(to_dims(in_v, sizeof(T), "softmax input", in));
    ANN_TRY(to_dims(out_v, sizeof(T), "softmax output", out));
    if (mask_v) {  // softmax.hpp:45-46
        ANN_TRY(to_dims(mask_v, sizeof(T), "maskedSoftmax mask", mask));
        if (!same_extents(in, out) || !same_extents(in, mask)) return fail(ANN_EINVAL, "maskedSoftmax shape mismatch.");
    }
    if (!same_extents(in, out)) return fail(ANN_EINVAL, "softmax shape mismatch.");  // softmax.hpp:29-30
    if (axis >= static_cast<uint32_t>(in.rank)) return fail(ANN_EINVAL, "softmax axis out of range.");
    if (causal && (qaxis >= static_cast<uint32_t>(in.rank) || kaxis >= static_cast<uint32_t>(in.rank)))
        return fail(ANN_EINVAL, "causalSoftmax query/key axis out of range.");
    if (in.numel() == 0) return ANN_OK;

    SoftmaxArgs a{};
    a.in = in.data;
    a.out = out.data;
    a.len = in.ext[axis];
    a.rows = in.numel() / a.len;
    a.s_in = in.str[axis];
    a.s_out = out.str[axis];
    a.outer.n = in.rank;
    for (int i = 0; i < in.rank; ++i) {
        a.outer.ext[i] = (i == static_cast<int>(axis)) ? 1 : in.ext[i];
        a.outer.sa[i] = in.str[i];
        a.outer.sb[i] = out.str[i];
    }
    a.causal = causal ? 1 : 0;
    a.q_is_axis = qaxis == axis;
    a.k_is_axis = kaxis == axis;
    auto component = [&](uint32_t ax, int64_t& div, int64_t& mod) {
        div = 1;
        for (int i = in.rank - 1; i > static_cast<int>(ax); --i) div *= a.outer.ext[i];
        mod = a.outer.ext[ax];
    };
    component(causal ? qaxis : 0, a.q_div, a.q_mod);
    component(causal ? kaxis : 0, a.k_div, a.k_mod);
    // Causal rows along the key axis keep [0, q]: the ring kernel copies only
    // that window when it is at most a quarter of the elements on average
    // (measured: [32,1,1024,4096], 1/8 kept, 0.203 -> 0.179 ms; square rows,
    // 1/2 kept, were slower windowed, 0.291 -> 0.341 ms, the window's index
    // arithmetic sitting on the copying warp's path).
    if (causal && a.k_is_axis && !a.q_is_axis) {
        double const tq = static_cast<double>(a.q_mod), n = static_cast<double>(a.len);
        double const kept = tq <= n ? tq * (tq + 1) / 2 : n * (n + 1) / 2 + (tq - n) * n;
        a.window = kept <= 0.25 * tq * n ? 1 : 0;
    }
    if (mask_v) {
        a.mask = mask.data;
        a.s_mask = mask.str[axis];
        a.mouter = a.outer;
        for (int i = 0; i < in.rank; ++i) a.mouter.sa[i] = mask.str[i];
    }
    // Equally spaced rows: the non-axis axes (extent > 1) merge into one, in
    // every operand, i.e. each one's stride is the next one's times its extent.
    {
        int prev = -1;
        bool uni = true;
        for (int i = 0; i < in.rank && uni; ++i) {
            if (i == static_cast<int>(axis) || in.ext[i] == 1) continue;
            if (prev >= 0) {
                uni = in.str[prev] == in.str[i] * in.ext[i] && out.str[prev] == out.str[i] * out.ext[i] &&
                      (!mask_v || mask.str[prev] == mask.str[i] * mask.ext[i]);
            }
            prev = i;
        }
        int last = -1;  // the innermost non-axis axis sets the row spacing
        for (int i = 0; i < in.rank; ++i)
            if (i != static_cast<int>(axis) && in.ext[i] != 1) last = i;
        a.uniform = uni ? 1 : 0;
        a.row_in = last >= 0 ? in.str[last] : 0;
        a.row_out = last >= 0 ? out.str[last] : 0;
        a.row_mask = (last >= 0 && mask_v) ? mask.str[last] : 0;
    }
    cudaStream_t s = as_stream(stream);
    char const* name = mask_v ? "maskedSoftmax" : causal ? "causalSoftmax" : "softmax";
    // 16-byte pieces: unit stride along the axis in every operand, the row
    // length a multiple of the piece, every row start 16-byte aligned.
    constexpr int NV = Vec16<T>::n;
    bool vec = a.s_in == 1 && a.s_out == 1 && a.len % NV == 0 && aligned(in.data, 16) && aligned(out.data, 16);
    if (mask_v) vec = vec && a.s_mask == 1 && aligned(mask.data, 16);
    for (int i = 0; vec && i < in.rank; ++i) {
        if (i == static_cast<int>(axis) || in.ext[i] == 1) continue;
        vec = in.str[i] % NV == 0 && out.str[i] % NV == 0 && (!mask_v || mask.str[i] % NV == 0);
    }
    // Up to 2048 elements a row stays in registers, 8 per lane: 1, 2, 4 or 8
    // warps per row; up to 8192 in the registers of a whole CTA, 16 or 32 per
    // lane; up to kSmemRowBytes in one CTA's shared memory. Longer rows stream
    // through L1/L2.
    int64_t const row_bytes = a.len * static_cast<int64_t>(sizeof(T));
    bool const smem_row = a.len > 8192 && row_bytes <= kSmemRowBytes;
    if (smem_row && row_bytes > (48 << 10)) {
        cudaError_t e = cudaSuccess;
        if (vec)
            e = cudaFuncSetAttribute(mask_v ? softmax_smem<T, NV, true> : softmax_smem<T, NV, false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemRowBytes));
        else
            e = cudaFuncSetAttribute(mask_v ? softmax_smem<T, 1, true> : softmax_smem<T, 1, false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemRowBytes));
        if (e != cudaSuccess) return fail(ANN_ECUDA, "softmax: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    }
    auto launch = [&](auto mask_tag) {
        constexpr bool M = decltype(mask_tag)::value;
        constexpr int CV = 8 / NV;  // 16-byte pieces per lane
        if (vec && a.len > 8192 && cluster_launched<T, M>(a, s)) {
            // quarter rows by bulk copy on clusters of four CTAs (softmax_cluster)
        } else if (vec && a.len > 8192 && bulk_launched<T, M>(a, s)) {
            // whole rows by bulk copy (softmax_bulk)
        } else if (smem_row) {
            size_t const bytes = static_cast<size_t>(row_bytes);
            if (vec) softmax_smem<T, NV, M><<<grid_for(a.rows, 1, 8), 256, bytes, s>>>(a);
            else softmax_smem<T, 1, M><<<grid_for(a.rows, 1, 8), 256, bytes, s>>>(a);
        } else if (vec && a.len <= 8192 && ring_launched<T, CV, M>(a, s)) {
            // rows through a bulk-copy ring (softmax_ring)
        } else if (vec) {
            if (a.len <= 256) softmax_regs<T, CV, NV, 1, M><<<grid_for(a.rows, 8), 256, 0, s>>>(a);
            else if (a.len <= 512) softmax_regs<T, CV, NV, 2, M><<<grid_for(a.rows, 4), 256, 0, s>>>(a);
            else if (a.len <= 1024) softmax_regs<T, CV, NV, 4, M><<<grid_for(a.rows, 2), 256, 0, s>>>(a);
            else if (a.len <= 2048) softmax_regs<T, CV, NV, 8, M><<<grid_for(a.rows, 1), 256, 0, s>>>(a);
            else if (a.len <= 4096) softmax_regs<T, 2 * CV, NV, 8, M><<<grid_for(a.rows, 1), 256, 0, s>>>(a);
            else if (a.len <= 8192) softmax_regs<T, 4 * CV, NV, 8, M><<<grid_for(a.rows, 1), 256, 0, s>>>(a);
            else softmax_kernel<T, 256, M><<<grid_for(a.rows, 1, 8), 256, 0, s>>>(a);
        } else {
            if (a.len <= 256) softmax_regs<T, 8, 1, 1, M><<<grid_for(a.rows, 8), 256, 0, s>>>(a);
            else if (a.len <= 512) softmax_regs<T, 8, 1, 2, M><<<grid_for(a.rows, 4), 256, 0, s>>>(a);
            else if (a.len <= 1024) softmax_regs<T, 8, 1, 4, M><<<grid_for(a.rows, 2), 256, 0, s>>>(a);
            else if (a.len <= 2048) softmax_regs<T, 8, 1, 8, M><<<grid_for(a.rows, 1), 256, 0, s>>>(a);
            else if (a.len <= 4096) softmax_regs<T, 16, 1, 8, M><<<grid_for(a.rows, 1), 256, 0, s>>>(a);
            else if (a.len <= 8192) softmax_regs<T, 32, 1, 8, M><<<grid_for(a.rows, 1), 256, 0, s>>>(a);
            else softmax_kernel<T, 256, M><<<grid_for(a.rows, 1, 8), 256, 0, s>>>(a);
        }
    };
    if (mask_v) launch(std::true_type{});
    else launch(std::false_type{});
    return check_launch(name);
}

// ---- ops::scale ----------------------------------------------------------
struct ScaleArgs {
    const void* in;
    void* out;
    int64_t n;
    Outer2 idx;  // all axes (generic path)
};

template <typename T, bool DENSE>
__global__ void __launch_bounds__(256) scale_kernel(ScaleArgs a, T scalar) {
    T const* in = static_cast<T const*>(a.in);
    T* out = static_cast<T*>(a.out);
    int64_t const step = static_cast<int64_t>(gridDim.x) * blockDim.x;
    int64_t const i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if constexpr (DENSE) {
        using V = typename Vec16<T>::type;
        constexpr int NV = Vec16<T>::n;
        int64_t const nv = a.n / NV;
        V const* iv = reinterpret_cast<V const*>(in);
        V* ov = reinterpret_cast<V*>(out);
        auto mul = [&](V v) {
            if constexpr (NV == 4) {
                v.x = v.x * scalar; v.y = v.y * scalar; v.z = v.z * scalar; v.w = v.w * scalar;
            } else {
                v.x = v.x * scalar; v.y = v.y * scalar;
            }
            return v;
        };
        int64_t i = i0;
        for (; i + step < nv; i += 2 * step) {  // two loads in flight
            V const v0 = iv[i], v1 = iv[i + step];
            ov[i] = mul(v0);
            ov[i + step] = mul(v1);
        }
        if (i < nv) ov[i] = mul(iv[i]);
        for (int64_t i = nv * NV + i0; i < a.n; i += step) out[i] = in[i] * scalar;
    } else {
        for (int64_t i = i0; i < a.n; i += step) {
            int64_t oi, oo;
            a.idx.offsets(i, oi, oo);
            out[oo] = in[oi] * scalar;
        }
    }
}

// Strided views whose innermost run is unit-stride in both tensors: one warp per
// row (the row's offsets decoded once), 16-byte vectors along the row.
struct ScaleRowArgs {
    const void* in;
    void* out;
    int64_t rows, len;  // len: elements per row, a multiple of the vector width
    Outer2 outer;       // axes outside the row
};

template <typename T>
__global__ void __launch_bounds__(256) scale_rows_kernel(ScaleRowArgs a, T scalar) {
    using V = typename Vec16<T>::type;
    constexpr int NV = Vec16<T>::n;
    int const lane = threadIdx.x & 31;
    int64_t const nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    int64_t const nvec = a.len / NV;
    for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < a.rows; r += nwarps) {
        int64_t oi, oo;
        a.outer.offsets(r, oi, oo);
        V const* src = reinterpret_cast<V const*>(static_cast<T const*>(a.in) + oi);
        V* dst = reinterpret_cast<V*>(static_cast<T*>(a.out) + oo);
        for (int64_t j = lane; j < nvec; j += 32) {
            V v = src[j];
            if constexpr (NV == 4) {
                v.x = v.x * scalar; v.y = v.y * scalar; v.z = v.z * scalar; v.w = v.w * scalar;
            } else {
                v.x = v.x * scalar; v.y = v.y * scalar;
            }
            dst[j] = v;
        }
    }
}

// Axes of (in, out) with extent 1 dropped and neighbours merged where both
// tensors are contiguous across them; returns the merged rank.
int merge_axes(const Dims& in, const Dims& out, int64_t* ext, int64_t* si, int64_t* so) {
    int r = 0;
    for (int i = 0; i < in.rank; ++i) {
        if (in.ext[i] == 1) continue;
        if (r > 0 && si[r - 1] == in.str[i] * in.ext[i] && so[r - 1] == out.str[i] * in.ext[i]) {
            ext[r - 1] *= in.ext[i];  // axis i continues the previous one in both tensors
            si[r - 1] = in.str[i];
            so[r - 1] = out.str[i];
            continue;
        }
        ext[r] = in.ext[i];
        si[r] = in.str[i];
        so[r] = out.str[i];
        ++r;
    }
    return r;
}

template <typename T>
int scale(ann_stream stream, const ann_view* in_v, T scalar, const ann_view* out_v) {
    Dims in, out;
    ANN_TRY(to_dims(in_v, sizeof(T), "scale input", in));
    ANN_TRY(to_dims(out_v, sizeof(T), "scale output", out));
    if (!same_extents(in, out)) return fail(ANN_EINVAL, "scale shape mismatch.");
    if (in.numel() == 0) return ANN_OK;
    ScaleArgs a{};
    a.in = in.data;
    a.out = out.data;
    a.n = in.numel();
    a.idx.n = in.rank;
    bool same = true;
    for (int i = 0; i < in.rank; ++i) {
        a.idx.ext[i] = in.ext[i];
        a.idx.sa[i] = in.str[i];
        a.idx.sb[i] = out.str[i];
        same = same && (in.ext[i] == 1 || in.str[i] == out.str[i]);
    }
    bool const dense = same && in.dense() && aligned(in.data, 16) && aligned(out.data, 16);
    if (!dense) {
        int64_t ext[ANN_MAX_RANK], si[ANN_MAX_RANK], so[ANN_MAX_RANK];
        int const r = merge_axes(in, out, ext, si, so);
        constexpr int NV = Vec16<T>::n;
        bool rows = r >= 1 && si[r - 1] == 1 && so[r - 1] == 1 && ext[r - 1] % NV == 0 && aligned(in.data, 16) &&
                    aligned(out.data, 16);
        for (int i = 0; rows && i < r - 1; ++i) rows = (si[i] * sizeof(T)) % 16 == 0 && (so[i] * sizeof(T)) % 16 == 0;
        if (rows) {
            ScaleRowArgs ra{};
            ra.in = in.data;
            ra.out = out.data;
            ra.len = ext[r - 1];
            ra.rows = a.n / ra.len;
            ra.outer.n = r - 1;
            for (int i = 0; i < r - 1; ++i) {
                ra.outer.ext[i] = ext[i];
                ra.outer.sa[i] = si[i];
                ra.outer.sb[i] = so[i];
            }
            int const blocks = static_cast<int>(std::min<int64_t>(ceil_div(ra.rows, 8), 148 * 16));
            scale_rows_kernel<T><<<blocks, 256, 0, as_stream(stream)>>>(ra, scalar);
            return check_launch("scale");
        }
    }
    int const grid = grid_for(a.n, 256 * 4);
    if (dense)
        scale_kernel<T, true><<<grid, 256, 0, as_stream(stream)>>>(a, scalar);
    else
        scale_kernel<T, false><<<grid, 256, 0, as_stream(stream)>>>(a, scalar);
    return check_launch("scale");
}

}  // namespace

int take_softmax_error(cudaStream_t s, uint32_t* bits) {
    unsigned int value = 0, zero = 0;
    if (cudaMemcpyFromSymbolAsync(&value, g_softmax_error, sizeof value, 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_softmax_error, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(ANN_ECUDA, "device error word: %s", cudaGetErrorString(cudaGetLastError()));
    *bits |= value;
    return ANN_OK;
}

}  // namespace ann

extern "C" {

int ann_softmax_f32(ann_stream s, const ann_view* in, const ann_view* out, uint32_t axis) {
    ANN_API_BEGIN
    return ann::softmax<float>(s, in, out, axis, false, 0, 0);
    ANN_API_END
}
int ann_softmax_f64(ann_stream s, const ann_view* in, const ann_view* out, uint32_t axis) {
    ANN_API_BEGIN
    return ann::softmax<double>(s, in, out, axis, false, 0, 0);
    ANN_API_END
}
int ann_causal_softmax_f32(ann_stream s, const ann_view* in, const ann_view* out, uint32_t axis, uint32_t qa,
                           uint32_t ka) {
    ANN_API_BEGIN
    return ann::softmax<float>(s, in, out, axis, true, qa, ka);
    ANN_API_END
}
int ann_causal_softmax_f64(ann_stream s, const ann_view* in, const ann_view* out, uint32_t axis, uint32_t qa,
                           uint32_t ka) {
    ANN_API_BEGIN
    return ann::softmax<double>(s, in, out, axis, true, qa, ka);
    ANN_API_END
}
int ann_masked_softmax_f32(ann_stream s, const ann_view* in, const ann_view* mask, const ann_view* out,
                           uint32_t axis) {
    ANN_API_BEGIN
    if (!mask) return ann::fail(ANN_EINVAL, "maskedSoftmax: mask is NULL.");
    return ann::softmax<float>(s, in, out, axis, false, 0, 0, mask);
    ANN_API_END
}

int ann_masked_softmax_f64(ann_stream s, const ann_view* in, const ann_view* mask, const ann_view* out,
                           uint32_t axis) {
    ANN_API_BEGIN
    if (!mask) return ann::fail(ANN_EINVAL, "maskedSoftmax: mask is NULL.");
    return ann::softmax<double>(s, in, out, axis, false, 0, 0, mask);
    ANN_API_END
}

int ann_scale_f32(ann_stream s, const ann_view* in, float scalar, const ann_view* out) {
    ANN_API_BEGIN
    return ann::scale<float>(s, in, scalar, out);
    ANN_API_END
}
int ann_scale_f64(ann_stream s, const ann_view* in, double scalar, const ann_view* out) {
    ANN_API_BEGIN
    return ann::scale<double>(s, in, scalar, out);
    ANN_API_END
}

}  // extern "C"
