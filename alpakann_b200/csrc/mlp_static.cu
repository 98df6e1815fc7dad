// mlp_static.cu -- the gated MLP for callers that must not allocate device
// memory while they run.
//
// Why: ann_mlp_* gets its two [batch, hidden] intermediate buffers from the
// caller's workspace or from cudaMallocAsync, and runs its GEMMs in cuBLAS,
// which may allocate workspace of its own. Some callers cannot allow any of
// that once they are running: a fixed device-memory budget decided at start-up,
// an allocator that must not be re-entered from this call site, a process
// that is not allowed to grow its footprint. This variant allocates nothing:
//  - the hidden activations live in one buffer that belongs to the library
//    image itself (a file-scope __device__ array of kScratchBytes), so no call
//    asks any allocator for memory;
//  - its two GEMMs are this file's own kernels, not a library's.
// The price is a size limit (kScratchBytes of hidden activations) and plain
// SIMT FMA GEMMs, slower than cuBLAS on large shapes.
//
// When the buffer is reserved: the CUDA runtime creates a module's __device__
// arrays when it loads the module on a device. Under lazy module loading (the
// default of CUDA 12 and what PyTorch sets) that is the first use of this
// file's code on the device, i.e. the first call of ann_mlp_static_scratch
// there; with CUDA_MODULE_LOADING=EAGER it is context creation. So the first
// call on each device takes kScratchBytes of device memory and later calls
// take none: make the first call at start-up, before a memory budget is fixed
// and before any stream capture. The memory stays reserved until the process
// exits.
//
// The first call on a device also looks the buffer's address up with
// cudaGetSymbolAddress (no allocation) and keeps it for that device ordinal
// for the life of the process; the kept address does not survive a
// cudaDeviceReset of that device. Nothing in the buffer has to start at zero:
// the first kernel writes every element the second one reads. There is one
// buffer per device: two calls whose kernels overlap on the GPU (different
// streams, no ordering between them) race on it.
#include <mutex>

#include "common.cuh"
#include "reduce.cuh"

namespace ann {
namespace {

constexpr size_t kScratchBytes = size_t{8} << 20;  // 8 MiB of hidden activations

static __device__ __align__(256) unsigned char g_mlp_scratch[kScratchBytes];

// Address of g_mlp_scratch on the current device, looked up once per device.
int scratch_address(void** out) {
    static std::mutex mu;
    static void* addr[128] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(ANN_ECUDA, "mlp (static scratch): cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 128) return fail(ANN_ENOTSUP, "mlp (static scratch): device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_mlp_scratch);
        if (e != cudaSuccess || !p)
            return fail(ANN_ECUDA, "mlp (static scratch): cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        addr[dev] = p;
    }
    *out = addr[dev];
    return ANN_OK;
}

constexpr int BM = 64, BN = 64, BK = 16, kThreads = 256;

struct GemmArgs {
    const void* x;   // [M, K], row pitch ldx (elements)
    const void* w0;  // [K, N], row pitch ldw0
    const void* w1;  // [K, N], row pitch ldw1 (GATED only)
    void* out;       // [M, N], row pitch ldo
    int64_t M, N, K, ldx, ldw0, ldw1, ldo;
};

// out = x . w0, or with GATED out = swiglu(x . w0, x . w1): 64x64 output tile
// per CTA, 16-deep K slices staged in shared memory, each thread 4x4 outputs
// (rows ty + 16 i, columns tx + 16 j), K ascending.
template <typename T, bool GATED>
__global__ void __launch_bounds__(kThreads) mlp_tile(GemmArgs a) {
    __shared__ T xs[BK][BM + 1];
    __shared__ T ws[GATED ? 2 : 1][BK][BN];
    T const* x = static_cast<T const*>(a.x);
    T const* w0 = static_cast<T const*>(a.w0);
    T const* w1 = static_cast<T const*>(a.w1);
    int const tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    int64_t const m0 = static_cast<int64_t>(blockIdx.y) * BM, n0 = static_cast<int64_t>(blockIdx.x) * BN;
    T acc0[4][4] = {}, acc1[4][4] = {};
    for (int64_t k0 = 0; k0 < a.K; k0 += BK) {
#pragma unroll
        for (int i = 0; i < BM * BK / kThreads; ++i) {
            int const idx = threadIdx.x + kThreads * i;
            int const m = idx / BK, k = idx % BK;
            bool const in = m0 + m < a.M && k0 + k < a.K;
            xs[k][m] = in ? x[(m0 + m) * a.ldx + k0 + k] : T(0);
        }
#pragma unroll
        for (int i = 0; i < BK * BN / kThreads; ++i) {
            int const idx = threadIdx.x + kThreads * i;
            int const k = idx / BN, n = idx % BN;
            bool const in = k0 + k < a.K && n0 + n < a.N;
            ws[0][k][n] = in ? w0[(k0 + k) * a.ldw0 + n0 + n] : T(0);
            if constexpr (GATED) ws[GATED ? 1 : 0][k][n] = in ? w1[(k0 + k) * a.ldw1 + n0 + n] : T(0);
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            T xv[4], wv0[4], wv1[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) xv[i] = xs[k][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                wv0[j] = ws[0][k][tx + 16 * j];
                if constexpr (GATED) wv1[j] = ws[GATED ? 1 : 0][k][tx + 16 * j];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc0[i][j] = fma(xv[i], wv0[j], acc0[i][j]);
                    if constexpr (GATED) acc1[i][j] = fma(xv[i], wv1[j], acc1[i][j]);
                }
        }
        __syncthreads();
    }
    T* out = static_cast<T*>(a.out);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int64_t const m = m0 + ty + 16 * i, n = n0 + tx + 16 * j;
            if (m >= a.M || n >= a.N) continue;
            T v = acc0[i][j];
            if constexpr (GATED) {  // swiglu: gate * sigmoid(gate) * up (elementwise.hpp:164-171)
                T const sig = T(1) / (T(1) + exp_t(-v));
                v = mul_rn(mul_rn(v, sig), acc1[i][j]);
            }
            out[m * a.ldo + n] = v;
        }
}

// Row pitch (elements) of a row-major view with unit column stride, or -1.
// An empty view has no elements to address: any pitch will do.
int64_t row_pitch(const Dims& d) {
    if (d.rank != 2) return -1;
    if (d.ext[0] == 0 || d.ext[1] == 0) return d.ext[1];
    if (d.ext[1] > 1 && d.str[1] != 1) return -1;
    if (d.ext[0] <= 1) return d.ext[1];
    return d.str[0] >= d.ext[1] ? d.str[0] : -1;
}

template <typename T>
int mlp_static(ann_stream stream, const ann_view* input, const ann_view* wgate, const ann_view* wup,
               const ann_view* wdown, const ann_view* output) {
    Dims in, g, u, d, o;
    ANN_TRY(to_dims(input, sizeof(T), "mlp input", in));
    ANN_TRY(to_dims(wgate, sizeof(T), "mlp Wgate", g));
    ANN_TRY(to_dims(wup, sizeof(T), "mlp Wup", u));
    ANN_TRY(to_dims(wdown, sizeof(T), "mlp Wdown", d));
    ANN_TRY(to_dims(output, sizeof(T), "mlp output", o));
    if (in.rank != 2 || g.rank != 2 || u.rank != 2 || d.rank != 2 || o.rank != 2)
        return fail(ANN_EINVAL, "gemm expects rank-2 operands.");
    if (g.ext[1] != u.ext[1]) return fail(ANN_EINVAL, "binaryOp shape mismatch.");
    if (g.ext[0] != in.ext[1] || u.ext[0] != in.ext[1] || d.ext[0] != g.ext[1] || o.ext[0] != in.ext[0] ||
        o.ext[1] != d.ext[1])
        return fail(ANN_EINVAL, "gemm shape mismatch.");
    int64_t const lx = row_pitch(in), lg = row_pitch(g), lu = row_pitch(u), ld = row_pitch(d), lo = row_pitch(o);
    if (lx < 0 || lg < 0 || lu < 0 || ld < 0 || lo < 0)
        return fail(ANN_EINVAL, "gemm expects row-major operands with unit column stride.");
    int64_t const M = in.ext[0], K = in.ext[1], F = g.ext[1], N = d.ext[1];
    uint64_t const need = static_cast<uint64_t>(M) * static_cast<uint64_t>(F) * sizeof(T);
    if (need > kScratchBytes)
        return fail(ANN_EINVAL,
                    "mlp (static scratch): the [batch, hidden] = [%lld, %lld] activations need %llu bytes, more "
                    "than the %zu bytes of static scratch; use ann_mlp_f32 / ann_mlp_f64.",
                    static_cast<long long>(M), static_cast<long long>(F), static_cast<unsigned long long>(need),
                    kScratchBytes);
    if (M == 0 || N == 0) return ANN_OK;
    if (ceil_div(M, BM) > 65535) return fail(ANN_ENOTSUP, "mlp (static scratch): batch too large for the grid.");
    void* hidden = nullptr;
    ANN_TRY(scratch_address(&hidden));
    cudaStream_t s = as_stream(stream);
    if (F > 0) {
        GemmArgs a{in.data, g.data, u.data, hidden, M, F, K, lx, lg, lu, F};
        mlp_tile<T, true><<<dim3(static_cast<unsigned>(ceil_div(F, BN)), static_cast<unsigned>(ceil_div(M, BM))),
                            kThreads, 0, s>>>(a);
        ANN_TRY(check_launch("mlp (static scratch) gate/up"));
    }
    GemmArgs b{hidden, d.data, nullptr, o.data, M, N, F, F, ld, 0, lo};
    mlp_tile<T, false><<<dim3(static_cast<unsigned>(ceil_div(N, BN)), static_cast<unsigned>(ceil_div(M, BM))),
                         kThreads, 0, s>>>(b);
    return check_launch("mlp (static scratch) down");
}

}  // namespace
}  // namespace ann

extern "C" int ann_mlp_static_scratch(ann_stream stream, int32_t dtype, const ann_view* input, const ann_view* wgate,
                                      const ann_view* wup, const ann_view* wdown, const ann_view* output) {
    ANN_API_BEGIN
    if (dtype == ANN_DTYPE_F32) return ann::mlp_static<float>(stream, input, wgate, wup, wdown, output);
    if (dtype == ANN_DTYPE_F64) return ann::mlp_static<double>(stream, input, wgate, wup, wdown, output);
    return ann::fail(ANN_EINVAL, "mlp (static scratch): dtype must be ANN_DTYPE_F32 or ANN_DTYPE_F64.");
    ANN_API_END
}
