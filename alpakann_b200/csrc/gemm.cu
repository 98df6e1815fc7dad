// gemm.cu -- gemm / qkvProjection (reference: onHost/matrix/gemm.hpp:28-33,
// onHost/nn/attention.hpp:38-52).
//
// The projection GEMMs stay on the vendor BLAS, as in the reference (which
// routes them to cuBLAS on CUDA through alpakaVendor). cuBLAS is loaded with
// dlopen at first use so the rest of the library does not depend on it.
// Row-major C[M,N] = A[M,K] * B[K,N] is issued as the column-major product
// C^T = B^T * A^T; the default (full FP32 / FP64) math mode is used.
#include <cublas_v2.h>
#include <dlfcn.h>

#include <map>
#include <mutex>

#include "common.cuh"

namespace ann {
namespace {

struct Cublas {
    decltype(&cublasCreate_v2) create = nullptr;
    decltype(&cublasSetStream_v2) set_stream = nullptr;
    decltype(&cublasSgemm_v2) sgemm = nullptr;
    decltype(&cublasDgemm_v2) dgemm = nullptr;
    bool ok = false;
};

Cublas& cublas() {
    static Cublas c;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libcublas.so.12", RTLD_NOW | RTLD_GLOBAL);
        if (h == nullptr) return;
        c.create = reinterpret_cast<decltype(c.create)>(dlsym(h, "cublasCreate_v2"));
        c.set_stream = reinterpret_cast<decltype(c.set_stream)>(dlsym(h, "cublasSetStream_v2"));
        c.sgemm = reinterpret_cast<decltype(c.sgemm)>(dlsym(h, "cublasSgemm_v2"));
        c.dgemm = reinterpret_cast<decltype(c.dgemm)>(dlsym(h, "cublasDgemm_v2"));
        c.ok = c.create && c.set_stream && c.sgemm && c.dgemm;
    });
    return c;
}

// One handle per (thread, device): cuBLAS handles must not be shared across
// threads that call concurrently.
int handle_for_current_device(cublasHandle_t& out) {
    thread_local std::map<int, cublasHandle_t> handles;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(ANN_ECUDA, "gemm: no CUDA device.");
    auto it = handles.find(dev);
    if (it == handles.end()) {
        cublasHandle_t h = nullptr;
        if (cublas().create(&h) != CUBLAS_STATUS_SUCCESS) return fail(ANN_ECUDA, "gemm: cublasCreate failed.");
        it = handles.emplace(dev, h).first;
    }
    out = it->second;
    return ANN_OK;
}

template <typename T>
int gemm(ann_stream stream, const ann_view* a_v, const ann_view* b_v, const ann_view* c_v, T beta = T(0)) {
    Dims a, b, c;
    ANN_TRY(to_dims(a_v, sizeof(T), "gemm A", a));
    ANN_TRY(to_dims(b_v, sizeof(T), "gemm B", b));
    ANN_TRY(to_dims(c_v, sizeof(T), "gemm C", c));
    if (a.rank != 2 || b.rank != 2 || c.rank != 2) return fail(ANN_EINVAL, "gemm expects rank-2 operands.");
    int64_t const M = a.ext[0], K = a.ext[1], N = b.ext[1];
    if (b.ext[0] != K || c.ext[0] != M || c.ext[1] != N) return fail(ANN_EINVAL, "gemm shape mismatch.");
    // A single row may carry any row pitch (a broadcast row has pitch 0).
    auto row_major = [](const Dims& d) {
        return (d.ext[1] <= 1 || d.str[1] == 1) && (d.ext[0] <= 1 || d.str[0] >= d.ext[1]);
    };
    if (!row_major(a) || !row_major(b) || !row_major(c))
        return fail(ANN_EINVAL, "gemm expects row-major operands with unit column stride.");
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail(ANN_ENOTSUP, "gemm: extents exceed int32.");
    if (M == 0 || N == 0) return ANN_OK;
    if (!cublas().ok) return fail(ANN_ENOTSUP, "gemm: libcublas.so.12 could not be loaded.");
    cublasHandle_t h;
    ANN_TRY(handle_for_current_device(h));
    if (cublas().set_stream(h, as_stream(stream)) != CUBLAS_STATUS_SUCCESS)
        return fail(ANN_ECUDA, "gemm: cublasSetStream failed.");
    T const one = 1;
    // Leading dimension of the column-major transpose: the row pitch, or the
    // row length when there is one row (its pitch is never used).
    auto ld = [](const Dims& d) {
        int64_t const l = d.ext[0] <= 1 ? d.ext[1] : d.str[0];
        return static_cast<int>(l > 0 ? l : 1);
    };
    int const lda = ld(a), ldb = ld(b), ldc = ld(c);
    cublasStatus_t st;
    if constexpr (sizeof(T) == 4)
        st = cublas().sgemm(h, CUBLAS_OP_N, CUBLAS_OP_N, static_cast<int>(N), static_cast<int>(M),
                            static_cast<int>(K), &one, static_cast<const float*>(b.data), ldb,
                            static_cast<const float*>(a.data), lda, &beta, static_cast<float*>(c.data), ldc);
    else
        st = cublas().dgemm(h, CUBLAS_OP_N, CUBLAS_OP_N, static_cast<int>(N), static_cast<int>(M),
                            static_cast<int>(K), &one, static_cast<const double*>(b.data), ldb,
                            static_cast<const double*>(a.data), lda, &beta, static_cast<double*>(c.data), ldc);
    if (st != CUBLAS_STATUS_SUCCESS) return fail(ANN_ECUDA, "gemm: cuBLAS status %d.", static_cast<int>(st));
    return ANN_OK;
}

template <typename T>
int qkv(ann_stream s, const ann_view* x, const ann_view* wq, const ann_view* wk, const ann_view* wv,
        const ann_view* q, const ann_view* k, const ann_view* v) {
    ANN_TRY(gemm<T>(s, x, wq, q));
    ANN_TRY(gemm<T>(s, x, wk, k));
    return gemm<T>(s, x, wv, v);
}

// output = residual + input . Wo: outputProjection (onHost/nn/attention.hpp:112-116)
// followed by ops::add (onHost/ops/elementwise.hpp:307-311) of the residual,
// the add done by the GEMM's epilogue (beta = 1) on an output that holds the
// residual (copied there first unless residual is output).
template <typename T>
int output_projection_residual(ann_stream s, const ann_view* in, const ann_view* wo, const ann_view* res,
                               const ann_view* out) {
    Dims r, o;
    ANN_TRY(to_dims(res, sizeof(T), "outputProjection residual", r));
    ANN_TRY(to_dims(out, sizeof(T), "outputProjection output", o));
    if (!same_extents(r, o)) return fail(ANN_EINVAL, "outputProjection residual shape mismatch.");
    bool same = r.data == o.data;
    for (int i = 0; same && i < r.rank; ++i) same = r.ext[i] <= 1 || r.str[i] == o.str[i];
    if (!same) {
        int const rc = sizeof(T) == 4 ? ann_scale_f32(s, res, 1.0f, out) : ann_scale_f64(s, res, 1.0, out);
        if (rc != ANN_OK) return rc;
    }
    return gemm<T>(s, in, wo, out, T(1));
}

}  // namespace
}  // namespace ann

extern "C" {

int ann_gemm_f32(ann_stream s, const ann_view* a, const ann_view* b, const ann_view* c) {
    ANN_API_BEGIN
    return ann::gemm<float>(s, a, b, c);
    ANN_API_END
}
int ann_gemm_f64(ann_stream s, const ann_view* a, const ann_view* b, const ann_view* c) {
    ANN_API_BEGIN
    return ann::gemm<double>(s, a, b, c);
    ANN_API_END
}
int ann_qkv_projection_f32(ann_stream s, const ann_view* x, const ann_view* wq, const ann_view* wk,
                           const ann_view* wv, const ann_view* q, const ann_view* k, const ann_view* v) {
    ANN_API_BEGIN
    return ann::qkv<float>(s, x, wq, wk, wv, q, k, v);
    ANN_API_END
}
int ann_qkv_projection_f64(ann_stream s, const ann_view* x, const ann_view* wq, const ann_view* wk,
                           const ann_view* wv, const ann_view* q, const ann_view* k, const ann_view* v) {
    ANN_API_BEGIN
    return ann::qkv<double>(s, x, wq, wk, wv, q, k, v);
    ANN_API_END
}

int ann_output_projection_residual_f32(ann_stream s, const ann_view* input, const ann_view* wo,
                                       const ann_view* residual, const ann_view* output) {
    ANN_API_BEGIN
    return ann::output_projection_residual<float>(s, input, wo, residual, output);
    ANN_API_END
}

int ann_output_projection_residual_f64(ann_stream s, const ann_view* input, const ann_view* wo,
                                       const ann_view* residual, const ann_view* output) {
    ANN_API_BEGIN
    return ann::output_projection_residual<double>(s, input, wo, residual, output);
    ANN_API_END
}

}  // extern "C"
