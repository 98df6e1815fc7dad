// common.cuh -- shared host/device helpers of the ann_b200 C ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <exception>
#include <string>

#include "ann_b200.h"

namespace ann {

// ---------------------------------------------------------------------------
// Errors: every entry point returns a code and leaves a thread-local message.
// ---------------------------------------------------------------------------
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

// After a launch: turn a pending CUDA error into ANN_ECUDA.
int check_launch(const char* what);

// Number of SMs of the current device (cached per device).
int sm_count();

// Device error words, one per translation unit that reports device-side
// errors: each reads its word on `s`, ORs it into *bits and clears it.
int take_embedding_error(cudaStream_t s, uint32_t* bits);
int take_decode_error(cudaStream_t s, uint32_t* bits);
int take_prefill_error(cudaStream_t s, uint32_t* bits);
int take_prefill_tc_error(cudaStream_t s, uint32_t* bits);
int take_prefill_tc2_error(cudaStream_t s, uint32_t* bits);
int take_selftest_error(cudaStream_t s, uint32_t* bits);
int take_rms_error(cudaStream_t s, uint32_t* bits);
int take_prefill_f64_error(cudaStream_t s, uint32_t* bits);
int take_softmax_error(cudaStream_t s, uint32_t* bits);
int take_multicast_error(cudaStream_t s, uint32_t* bits);
int take_attention_tc_error(cudaStream_t s, uint32_t* bits);

// ---------------------------------------------------------------------------
// Views: ann_view with byte pitches -> element strides, validated.
// ---------------------------------------------------------------------------
struct Dims {
    int rank = 0;
    int64_t ext[ANN_MAX_RANK] = {};
    int64_t str[ANN_MAX_RANK] = {};  // element strides
    void* data = nullptr;

    int64_t numel() const {
        int64_t n = 1;
        for (int a = 0; a < rank; ++a) n *= ext[a];
        return n;
    }
    // Strides of a dense row-major tensor of these extents?
    bool dense() const {
        int64_t expect = 1;
        for (int a = rank - 1; a >= 0; --a) {
            if (ext[a] != 1 && str[a] != expect) return false;
            expect *= ext[a];
        }
        return true;
    }
};

// Converts and checks a view: non-null descriptor, rank in [1, ANN_MAX_RANK],
// non-negative extents, pitches non-negative multiples of elem_bytes, data
// non-null unless the view is empty.
int to_dims(const ann_view* v, size_t elem_bytes, const char* what, Dims& out);

inline bool same_extents(const Dims& a, const Dims& b) {
    if (a.rank != b.rank) return false;
    for (int i = 0; i < a.rank; ++i)
        if (a.ext[i] != b.ext[i]) return false;
    return true;
}

std::string extents_str(const Dims& d);

inline bool aligned(const void* p, size_t bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

inline cudaStream_t as_stream(ann_stream s) { return reinterpret_cast<cudaStream_t>(s); }

// Offsets of a multi-index over the leading `n` axes for up to two tensors
// that share extents (row enumeration of row-wise kernels).
struct Outer2 {
    int n = 0;
    int64_t ext[ANN_MAX_RANK] = {};
    int64_t sa[ANN_MAX_RANK] = {};
    int64_t sb[ANN_MAX_RANK] = {};

    __host__ __device__ inline void offsets(int64_t flat, int64_t& oa, int64_t& ob) const {
        oa = 0;
        ob = 0;
        for (int a = n - 1; a >= 0; --a) {
            int64_t const i = flat % ext[a];
            flat /= ext[a];
            oa += i * sa[a];
            ob += i * sb[a];
        }
    }
};

template <typename T>
struct Vec16;  // 16-byte vector of T
template <>
struct Vec16<float> {
    using type = float4;
    static constexpr int n = 4;
};
template <>
struct Vec16<double> {
    using type = double2;
    static constexpr int n = 2;
};

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// (batch, head) pairs per dispatch chunk of a prefill grid: as many as keep one
// chunk's K+V within 32 MiB of L2, but at least two waves of CTAs per chunk
// (`resident` CTAs per SM), so that longest-first inside a chunk still fills
// the GPU. A chunk of all pairs means one global longest-first order.
inline int64_t head_chunk_for(int64_t bhs, int64_t q_tiles, int64_t kv_bytes_per_head, int resident) {
    int64_t chunk = kv_bytes_per_head > 0 ? (int64_t{32} << 20) / kv_bytes_per_head : bhs;
    int64_t const waves = ceil_div(int64_t{2} * sm_count() * resident, q_tiles > 0 ? q_tiles : 1);
    if (chunk < waves) chunk = waves;
    if (chunk < 1) chunk = 1;
    if (chunk >= bhs) return bhs;
    return ceil_div(bhs, ceil_div(bhs, chunk));  // chunks of equal size: no short last chunk
}

inline int grid_for(int64_t work_items, int per_block, int max_blocks_per_sm = 16) {
    int64_t blocks = ceil_div(work_items, per_block);
    int64_t cap = static_cast<int64_t>(sm_count()) * max_blocks_per_sm;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return static_cast<int>(blocks);
}

}  // namespace ann

// Entry-point boilerplate: catch C++ exceptions at the C boundary.
#define ANN_API_BEGIN \
    ann::clear_error(); \
    try {
#define ANN_API_END                                                       \
    }                                                                     \
    catch (std::exception const& e) {                                     \
        return ann::fail(ANN_EINVAL, "%s", e.what());                     \
    }                                                                     \
    catch (...) {                                                         \
        return ann::fail(ANN_EINVAL, "unknown C++ exception");            \
    }

#define ANN_TRY(expr)                 \
    do {                              \
        int ann_rc__ = (expr);        \
        if (ann_rc__ != ANN_OK) return ann_rc__; \
    } while (0)
