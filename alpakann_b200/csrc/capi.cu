// capi.cu -- library-level entry points and host helpers shared by all ops.
#include <cstdarg>
#include <mutex>
#include <sstream>
#include <stdexcept>

#include "common.cuh"

namespace ann {

namespace {
thread_local std::string g_last_error;
}

void clear_error() { g_last_error.clear(); }

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int check_launch(const char* what) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return fail(ANN_ECUDA, "%s: %s", what, cudaGetErrorString(err));
    return ANN_OK;
}

int sm_count() {
    static std::mutex mu;
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

std::string extents_str(const Dims& d) {
    std::ostringstream os;
    os << "{";
    for (int i = 0; i < d.rank; ++i) os << (i ? ", " : "") << d.ext[i];
    os << "}";
    return os.str();
}

int to_dims(const ann_view* v, size_t elem_bytes, const char* what, Dims& out) {
    if (v == nullptr) return fail(ANN_EINVAL, "%s: view descriptor is NULL.", what);
    if (v->rank < 1 || v->rank > ANN_MAX_RANK) return fail(ANN_EINVAL, "%s: rank %d out of range.", what, v->rank);
    out.rank = v->rank;
    out.data = v->data;
    bool empty = false;
    for (int a = 0; a < v->rank; ++a) {
        if (v->extents[a] < 0) return fail(ANN_EINVAL, "%s: negative extent on axis %d.", what, a);
        if (v->pitches[a] < 0 || v->pitches[a] % static_cast<int64_t>(elem_bytes) != 0)
            return fail(ANN_EINVAL, "%s: pitch %lld of axis %d is not a non-negative multiple of %zu bytes.", what,
                        static_cast<long long>(v->pitches[a]), a, elem_bytes);
        out.ext[a] = v->extents[a];
        out.str[a] = v->pitches[a] / static_cast<int64_t>(elem_bytes);
        empty = empty || v->extents[a] == 0;
    }
    if (!empty && v->data == nullptr) return fail(ANN_EINVAL, "%s: data pointer is NULL.", what);
    if (!empty && !aligned(v->data, elem_bytes)) return fail(ANN_EINVAL, "%s: data pointer is misaligned.", what);
    return ANN_OK;
}

}  // namespace ann

extern "C" {

int ann_version(void) { return ANN_B200_VERSION; }

const char* ann_last_error(void) { return ann::g_last_error.c_str(); }

int ann_take_device_error(ann_stream stream, uint32_t* bits) {
    ann::clear_error();
    if (bits == nullptr) return ann::fail(ANN_EINVAL, "ann_take_device_error: bits is NULL.");
    uint32_t value = 0;
    cudaStream_t s = ann::as_stream(stream);
    ANN_TRY(ann::take_embedding_error(s, &value));
    ANN_TRY(ann::take_decode_error(s, &value));
    ANN_TRY(ann::take_prefill_error(s, &value));
    ANN_TRY(ann::take_prefill_tc_error(s, &value));
    ANN_TRY(ann::take_prefill_tc2_error(s, &value));
    ANN_TRY(ann::take_selftest_error(s, &value));
    ANN_TRY(ann::take_rms_error(s, &value));
    ANN_TRY(ann::take_prefill_f64_error(s, &value));
    ANN_TRY(ann::take_softmax_error(s, &value));
    ANN_TRY(ann::take_multicast_error(s, &value));
    ANN_TRY(ann::take_attention_tc_error(s, &value));
    *bits = value;
    return ANN_OK;
}

}  // extern "C"
