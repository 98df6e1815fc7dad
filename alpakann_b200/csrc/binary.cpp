// binary.cpp -- flat model artifacts ("neural-bunch model format v1") to
// device memory, and the SHA-256 digest that guards them.
//
// Reference: include/alpaka/nn/onHost/core/binary.hpp (TensorSpec :33-39,
// sha256File :212-232, loadBinaryTensor :234-323).
//
//  - SHA-256 is FIPS 180-4. The round constants and the initial hash value are
//    not typed in: they are computed at start-up from their definition (the
//    first 32 fractional bits of the cube roots of the first 64 primes and of
//    the square roots of the first 8), with exact integer roots. Blocks are
//    compressed with the x86 SHA extensions where the CPU has them (about
//    2 GB/s per core) and by the scalar recurrence elsewhere; both give the
//    same digest.
//  - A load validates everything the reference validates, in the same order
//    and with the same messages, before it reads the payload. The payload then
//    streams through two pinned staging buffers: while the copy engine moves
//    chunk i to the device, several host threads read chunk i+1 from the file.
//    The reference reads the whole tensor into one host allocation first.
//  - ann_load_binary_tensor_box loads one rank's rectangle of a row-major
//    matrix (a column-parallel Wq/Wk/Wv shard, a row-parallel Wo shard)
//    without reading the rest of the rows.
#include <cpuid.h>
#include <fcntl.h>
#include <immintrin.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <limits>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

namespace {

// ---------------------------------------------------------------------------
// SHA-256 constants from their definition.
// ---------------------------------------------------------------------------
using u128 = unsigned __int128;

// floor(v^(1/k)) for k = 2 or 3, by bisection on exact 128-bit integers.
uint64_t iroot(u128 v, int k) {
    uint64_t lo = 0, hi = uint64_t{1} << (k == 2 ? 63 : 42);
    while (lo < hi) {
        uint64_t const mid = lo + (hi - lo + 1) / 2;
        u128 p = mid;
        for (int i = 1; i < k; ++i) p *= mid;
        if (p <= v)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

struct Sha256Constants {
    uint32_t k[64];
    uint32_t h0[8];
    Sha256Constants() {
        int primes[64];
        int n = 0;
        for (int c = 2; n < 64; ++c) {
            bool prime = true;
            for (int d = 2; d * d <= c; ++d)
                if (c % d == 0) prime = false;
            if (prime) primes[n++] = c;
        }
        // frac(cbrt(p)) * 2^32 = floor(cbrt(p * 2^96)) mod 2^32, and
        // frac(sqrt(p)) * 2^32 = floor(sqrt(p * 2^64)) mod 2^32.
        for (int i = 0; i < 64; ++i) k[i] = static_cast<uint32_t>(iroot(static_cast<u128>(primes[i]) << 96, 3));
        for (int i = 0; i < 8; ++i) h0[i] = static_cast<uint32_t>(iroot(static_cast<u128>(primes[i]) << 64, 2));
    }
};

Sha256Constants const& constants() {
    static Sha256Constants const c;
    return c;
}

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

inline uint32_t load_be32(uint8_t const* p) {
    return (uint32_t{p[0]} << 24) | (uint32_t{p[1]} << 16) | (uint32_t{p[2]} << 8) | uint32_t{p[3]};
}

// FIPS 180-4 section 6.2.2, one 64-byte block at a time.
void compress_scalar(uint32_t state[8], uint8_t const* data, size_t blocks) {
    uint32_t const* K = constants().k;
    for (; blocks != 0; --blocks, data += 64) {
        uint32_t w[64];
        for (int t = 0; t < 16; ++t) w[t] = load_be32(data + 4 * t);
        for (int t = 16; t < 64; ++t) {
            uint32_t const x = w[t - 15], y = w[t - 2];
            uint32_t const sigma0 = rotr(x, 7) ^ rotr(x, 18) ^ (x >> 3);
            uint32_t const sigma1 = rotr(y, 17) ^ rotr(y, 19) ^ (y >> 10);
            w[t] = w[t - 16] + sigma0 + w[t - 7] + sigma1;
        }
        uint32_t v[8];
        for (int i = 0; i < 8; ++i) v[i] = state[i];
        for (int t = 0; t < 64; ++t) {
            uint32_t const a = v[0], e = v[4];
            uint32_t const big1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
            uint32_t const ch = (e & v[5]) ^ (~e & v[6]);
            uint32_t const t1 = v[7] + big1 + ch + K[t] + w[t];
            uint32_t const big0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
            uint32_t const maj = (a & v[1]) ^ (a & v[2]) ^ (v[1] & v[2]);
            for (int i = 7; i > 0; --i) v[i] = v[i - 1];
            v[4] += t1;
            v[0] = t1 + big0 + maj;
        }
        for (int i = 0; i < 8; ++i) state[i] += v[i];
    }
}

// The same compression on the SHA extensions. sha256rnds2 runs two rounds on
// the state split as (A,B,E,F) and (C,D,G,H); after two rounds the new
// (C,D,G,H) is the old (A,B,E,F), so the two halves swap roles every call.
// sha256msg1/msg2 plus one alignr produce four schedule words W[t..t+3].
__attribute__((target("sha,sse4.1,ssse3"))) void compress_shani(uint32_t state[8], uint8_t const* data,
                                                                 size_t blocks) {
    uint32_t const* K = constants().k;
    __m128i const bswap = _mm_set_epi8(12, 13, 14, 15, 8, 9, 10, 11, 4, 5, 6, 7, 0, 1, 2, 3);
    __m128i abef = _mm_set_epi32(static_cast<int>(state[0]), static_cast<int>(state[1]), static_cast<int>(state[4]),
                                 static_cast<int>(state[5]));
    __m128i cdgh = _mm_set_epi32(static_cast<int>(state[2]), static_cast<int>(state[3]), static_cast<int>(state[6]),
                                 static_cast<int>(state[7]));
    for (; blocks != 0; --blocks, data += 64) {
        __m128i const abef0 = abef, cdgh0 = cdgh;
        __m128i m[4];
        for (int i = 0; i < 4; ++i)
            m[i] = _mm_shuffle_epi8(_mm_loadu_si128(reinterpret_cast<__m128i const*>(data + 16 * i)), bswap);
        for (int g = 0; g < 16; ++g) {  // rounds 4g .. 4g+3
            if (g >= 4) {
                // m[g%4] holds W[4g-16..], m[(g+1)%4] W[4g-12..], m[(g+2)%4] W[4g-8..], m[(g+3)%4] W[4g-4..]
                __m128i w = _mm_sha256msg1_epu32(m[g & 3], m[(g + 1) & 3]);
                w = _mm_add_epi32(w, _mm_alignr_epi8(m[(g + 3) & 3], m[(g + 2) & 3], 4));
                m[g & 3] = _mm_sha256msg2_epu32(w, m[(g + 3) & 3]);
            }
            __m128i wk = _mm_add_epi32(m[g & 3], _mm_loadu_si128(reinterpret_cast<__m128i const*>(K + 4 * g)));
            cdgh = _mm_sha256rnds2_epu32(cdgh, abef, wk);
            wk = _mm_shuffle_epi32(wk, 0x0E);
            abef = _mm_sha256rnds2_epu32(abef, cdgh, wk);
        }
        abef = _mm_add_epi32(abef, abef0);
        cdgh = _mm_add_epi32(cdgh, cdgh0);
    }
    state[0] = static_cast<uint32_t>(_mm_extract_epi32(abef, 3));
    state[1] = static_cast<uint32_t>(_mm_extract_epi32(abef, 2));
    state[4] = static_cast<uint32_t>(_mm_extract_epi32(abef, 1));
    state[5] = static_cast<uint32_t>(_mm_extract_epi32(abef, 0));
    state[2] = static_cast<uint32_t>(_mm_extract_epi32(cdgh, 3));
    state[3] = static_cast<uint32_t>(_mm_extract_epi32(cdgh, 2));
    state[6] = static_cast<uint32_t>(_mm_extract_epi32(cdgh, 1));
    state[7] = static_cast<uint32_t>(_mm_extract_epi32(cdgh, 0));
}

bool cpu_has_sha() {
    unsigned a, b, c, d;
    if (!__get_cpuid(1, &a, &b, &c, &d)) return false;
    bool const ssse3 = c & (1u << 9), sse41 = c & (1u << 19);
    if (!__get_cpuid_count(7, 0, &a, &b, &c, &d)) return false;
    return ssse3 && sse41 && (b & (1u << 29));
}

using CompressFn = void (*)(uint32_t*, uint8_t const*, size_t);

CompressFn compress_fn() {
    static CompressFn const fn = [] {
        char const* env = std::getenv("ANN_SHA256_SCALAR");
        bool const scalar = env && *env && *env != '0';
        return (!scalar && cpu_has_sha()) ? &compress_shani : &compress_scalar;
    }();
    return fn;
}

struct Sha256 {
    uint32_t state[8];
    uint8_t pending[64];
    size_t pending_len = 0;
    uint64_t total = 0;
    CompressFn compress = compress_fn();

    Sha256() { std::memcpy(state, constants().h0, sizeof(state)); }

    void update(uint8_t const* p, size_t n) {
        total += n;
        if (pending_len != 0) {
            size_t const take = std::min(n, size_t{64} - pending_len);
            std::memcpy(pending + pending_len, p, take);
            pending_len += take;
            p += take;
            n -= take;
            if (pending_len < 64) return;
            compress(state, pending, 1);
            pending_len = 0;
        }
        size_t const blocks = n / 64;
        if (blocks != 0) compress(state, p, blocks);
        p += 64 * blocks;
        n -= 64 * blocks;
        std::memcpy(pending, p, n);
        pending_len = n;
    }

    // Padding: 0x80, zeros up to 56 mod 64, the bit length big-endian.
    void hex(char out[65]) {
        uint64_t const bits = total * 8;
        uint8_t tail[128] = {};
        std::memcpy(tail, pending, pending_len);
        tail[pending_len] = 0x80;
        size_t const len = pending_len < 56 ? 64 : 128;
        for (int i = 0; i < 8; ++i) tail[len - 1 - i] = static_cast<uint8_t>(bits >> (8 * i));
        compress(state, tail, len / 64);
        static char const digits[] = "0123456789abcdef";
        for (int i = 0; i < 8; ++i)
            for (int j = 0; j < 8; ++j) out[8 * i + j] = digits[(state[i] >> (28 - 4 * j)) & 0xF];
        out[64] = '\0';
    }
};

// ---------------------------------------------------------------------------
// Files.
// ---------------------------------------------------------------------------
struct Fd {
    int fd = -1;
    explicit Fd(char const* path) : fd(::open(path, O_RDONLY | O_CLOEXEC)) {}
    ~Fd() {
        if (fd >= 0) ::close(fd);
    }
    Fd(Fd const&) = delete;
    Fd& operator=(Fd const&) = delete;
};

// Reads exactly n bytes at `offset`; false on an error or end of file.
bool pread_full(int fd, void* dst, size_t n, uint64_t offset) {
    char* p = static_cast<char*>(dst);
    while (n != 0) {
        ssize_t const r = ::pread(fd, p, n, static_cast<off_t>(offset));
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;
        p += r;
        n -= static_cast<size_t>(r);
        offset += static_cast<uint64_t>(r);
    }
    return true;
}

constexpr size_t kHashChunk = size_t{4} << 20;

int sha256_of(char const* path, char out[65]) {
    Fd f(path);
    if (f.fd < 0) return ann::fail(ANN_EIO, "sha256File: cannot open '%s'.", path);
    struct stat st {};
    if (::fstat(f.fd, &st) != 0 || S_ISDIR(st.st_mode))
        return ann::fail(ANN_EIO, "sha256File: read error in '%s'.", path);
    ::posix_fadvise(f.fd, 0, 0, POSIX_FADV_SEQUENTIAL);
    std::string buf(kHashChunk, '\0');
    Sha256 sha;
    uint64_t offset = 0;
    for (;;) {
        ssize_t const r = ::pread(f.fd, buf.data(), buf.size(), static_cast<off_t>(offset));
        if (r < 0 && errno == EINTR) continue;
        if (r < 0) return ann::fail(ANN_EIO, "sha256File: read error in '%s'.", path);
        if (r == 0) break;
        sha.update(reinterpret_cast<uint8_t const*>(buf.data()), static_cast<size_t>(r));
        offset += static_cast<uint64_t>(r);
    }
    sha.hex(out);
    return ANN_OK;
}

// ---------------------------------------------------------------------------
// Readers: a chunk is read by several threads at once. One thread copies from
// the page cache at about 10 GB/s, a fifth of what the copy engine takes from
// pinned memory; the workers of this pool (created at first use, alive for
// the process) and the calling thread split each chunk between them.
// ANN_LOAD_THREADS overrides the thread count (1 = the calling thread only).
// ---------------------------------------------------------------------------
class Readers {
public:
    static Readers& get() {
        static Readers* r = new Readers;  // never destroyed: workers sleep until process exit
        return *r;
    }
    int threads() const { return static_cast<int>(workers_) + 1; }

    // Runs fn(part) for every part in [0, parts); returns when all are done.
    // One job at a time (callers hold the staging lock).
    void run(int parts, std::function<void(int)> const& fn) {
        if (parts <= 1 || workers_ == 0) {
            for (int p = 0; p < parts; ++p) fn(p);
            return;
        }
        uint64_t gen;
        {
            std::lock_guard<std::mutex> lock(mu_);
            gen = ++generation_;
            job_.store(&fn);
            parts_.store(parts);
            left_ = parts;
            claim_.store(gen << 32);  // (generation, next part) -- published last
        }
        wake_.notify_all();
        work(gen);
        std::unique_lock<std::mutex> lock(mu_);
        done_.wait(lock, [&] { return left_ == 0; });
    }

private:
    Readers() {
        unsigned const hc = std::thread::hardware_concurrency();
        int n = static_cast<int>(std::min(8u, std::max(1u, hc / 2)));
        if (char const* env = std::getenv("ANN_LOAD_THREADS")) n = std::max(1, std::atoi(env));
        workers_ = static_cast<unsigned>(n - 1);
        for (unsigned i = 0; i < workers_; ++i) std::thread([this] { loop(); }).detach();
    }
    // Claims parts of job `gen` until none is left. A part is claimed by a
    // compare-exchange on (generation, next part), so a thread that woke for
    // an older job can never claim a part of a newer one; and a job cannot
    // finish (nor its fn / parts change) while a claimed part is running.
    void work(uint64_t gen) {
        for (;;) {
            uint64_t v = claim_.load();
            if ((v >> 32) != gen) return;
            if (static_cast<int>(v & 0xffffffffu) >= parts_.load()) return;
            if (!claim_.compare_exchange_weak(v, v + 1)) continue;
            (*job_.load())(static_cast<int>(v & 0xffffffffu));
            std::lock_guard<std::mutex> lock(mu_);
            if (--left_ == 0) done_.notify_all();
        }
    }
    void loop() {
        uint64_t seen = 0;
        for (;;) {
            uint64_t gen;
            {
                std::unique_lock<std::mutex> lock(mu_);
                wake_.wait(lock, [&] { return generation_ != seen; });
                seen = gen = generation_;
            }
            work(gen);
        }
    }
    unsigned workers_ = 0;
    std::mutex mu_;
    std::condition_variable wake_, done_;
    std::atomic<std::function<void(int)> const*> job_{nullptr};
    std::atomic<int> parts_{0};
    std::atomic<uint64_t> claim_{0};
    int left_ = 0;            // guarded by mu_
    uint64_t generation_ = 0;  // guarded by mu_
};

// ---------------------------------------------------------------------------
// Pinned staging: two buffers shared by all loads of the process. Each buffer
// carries the event of the last copy that read it; a load waits on that event
// before it writes the buffer again, so a load may return while its last copy
// is still in flight on the caller's stream.
// ---------------------------------------------------------------------------
constexpr size_t kStageBytes = size_t{16} << 20;

struct Staging {
    std::mutex mu;
    void* buf[2] = {nullptr, nullptr};
    cudaEvent_t busy[2] = {nullptr, nullptr};  // created on the device of the copy that recorded it

    int acquire() {
        for (int i = 0; i < 2; ++i)
            if (!buf[i] && cudaHostAlloc(&buf[i], kStageBytes, cudaHostAllocPortable) != cudaSuccess) {
                buf[i] = nullptr;
                return ann::fail(ANN_ECUDA, "loadBinaryTensor: cannot allocate %zu bytes of pinned staging memory",
                                 kStageBytes);
            }
        return ANN_OK;
    }
    int wait(int i) {
        if (!busy[i]) return ANN_OK;
        cudaError_t const e = cudaEventSynchronize(busy[i]);
        cudaEventDestroy(busy[i]);
        busy[i] = nullptr;
        if (e != cudaSuccess) return ann::fail(ANN_ECUDA, "loadBinaryTensor: staging copy failed: %s", cudaGetErrorString(e));
        return ANN_OK;
    }
    int mark(int i, cudaStream_t s) {
        if (cudaEventCreateWithFlags(&busy[i], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventRecord(busy[i], s) != cudaSuccess) {
            // Without an event the next user of this buffer cannot know when
            // the copy has read it: wait for the copy here.
            if (busy[i]) cudaEventDestroy(busy[i]);
            busy[i] = nullptr;
            cudaStreamSynchronize(s);
            return ann::fail(ANN_ECUDA, "loadBinaryTensor: cannot record the staging event");
        }
        return ANN_OK;
    }
};

Staging& staging() {
    static Staging* s = new Staging;  // never destroyed: copies may outlive static destruction order
    return *s;
}

std::string lower(std::string v) {
    for (char& c : v)
        if (c >= 'A' && c <= 'Z') c = static_cast<char>(c - 'A' + 'a');
    return v;
}

// Checks of loadBinaryTensor (onHost/core/binary.hpp:263-305) in the
// reference's order. On success *byte_count is count * element_size.
int validate(char const* path, ann_tensor_spec const* spec, size_t element_size, char const* expected_sha256,
             uint64_t* byte_count) {
    if (!path) return ann::fail(ANN_EINVAL, "loadBinaryTensor: path is NULL.");
    if (!spec) return ann::fail(ANN_EINVAL, "loadBinaryTensor: spec is NULL.");
    if (element_size != 4 && element_size != 8)
        return ann::fail(ANN_EINVAL, "loadBinaryTensor supports only float32 and float64 tensors.");
    char const* name = spec->name ? spec->name : "";
    if (spec->count == 0) return ann::fail(ANN_EINVAL, "loadBinaryTensor: tensor '%s' has zero elements.", name);
    if (spec->shape_rank < 0 || (spec->shape_rank > 0 && !spec->shape))
        return ann::fail(ANN_EINVAL, "loadBinaryTensor: shape of tensor '%s' is malformed.", name);
    if (spec->shape_rank > 0) {
        uint64_t product = 1;
        for (int i = 0; i < spec->shape_rank; ++i) {
            uint64_t const e = spec->shape[i];
            if (e != 0 && product > std::numeric_limits<uint64_t>::max() / e)
                return ann::fail(ANN_EINVAL, "loadBinaryTensor: shape of tensor '%s' overflows std::size_t.", name);
            product *= e;
        }
        if (product != spec->count)
            return ann::fail(ANN_EINVAL,
                             "loadBinaryTensor: shape product %llu of tensor '%s' does not match count %llu.",
                             static_cast<unsigned long long>(product), name,
                             static_cast<unsigned long long>(spec->count));
    }
    struct stat st {};
    if (::stat(path, &st) != 0)
        return ann::fail(ANN_EIO, "loadBinaryTensor: cannot stat '%s': %s", path, std::strerror(errno));
    if (!S_ISREG(st.st_mode))
        return ann::fail(ANN_EIO, "loadBinaryTensor: cannot stat '%s': not a regular file", path);
    uint64_t const file_size = static_cast<uint64_t>(st.st_size);
    if (spec->offset_bytes % 64 != 0)
        return ann::fail(ANN_EINVAL, "loadBinaryTensor: offset %llu of tensor '%s' is not 64-byte aligned.",
                         static_cast<unsigned long long>(spec->offset_bytes), name);
    if (spec->count > std::numeric_limits<uint64_t>::max() / element_size)
        return ann::fail(ANN_EINVAL, "loadBinaryTensor: byte size of tensor '%s' overflows std::size_t.", name);
    uint64_t const bytes = spec->count * element_size;
    if (spec->offset_bytes > file_size || bytes > file_size - spec->offset_bytes)
        return ann::fail(ANN_EINVAL,
                         "loadBinaryTensor: tensor '%s' (%llu bytes at offset %llu) exceeds file size %llu.", name,
                         static_cast<unsigned long long>(bytes), static_cast<unsigned long long>(spec->offset_bytes),
                         static_cast<unsigned long long>(file_size));
    if (expected_sha256 && *expected_sha256) {
        char actual[65];
        ANN_TRY(sha256_of(path, actual));
        if (lower(expected_sha256) != actual)
            return ann::fail(ANN_EIO, "loadBinaryTensor: SHA-256 mismatch for '%s': expected %s, got %s.", path,
                             expected_sha256, actual);
    }
    *byte_count = bytes;
    return ANN_OK;
}

// Streams `rows` rows of `seg` bytes each to the device. Row r of the file
// starts at file_off + r * file_pitch; row r of the destination at
// dst + r * dst_pitch. Rows are packed `seg` bytes apart in staging; when
// file_pitch == seg (whole rows, contiguous in the file) a chunk is one read,
// else one read per row.
int stream_rows(cudaStream_t s, int fd, char const* path, char const* name, uint64_t file_off, uint64_t file_pitch,
                uint64_t seg, uint64_t rows, char* dst, uint64_t dst_pitch) {
    Staging& st = staging();
    std::lock_guard<std::mutex> lock(st.mu);
    ANN_TRY(st.acquire());
    bool const contiguous_src = file_pitch == seg;
    bool const contiguous_dst = dst_pitch == seg;
    // A 1-D run (both sides contiguous) is chunked by bytes; otherwise by rows.
    uint64_t const total = seg * rows;
    uint64_t const rows_per_chunk = seg >= kStageBytes ? 0 : kStageBytes / seg;
    if (!(contiguous_src && contiguous_dst) && rows_per_chunk == 0)
        return ann::fail(ANN_ENOTSUP, "loadBinaryTensor: a row of %llu bytes exceeds the %zu-byte staging buffer",
                         static_cast<unsigned long long>(seg), kStageBytes);
    uint64_t done_rows = 0, done_bytes = 0;
    for (int chunk = 0;; ++chunk) {
        int const b = chunk & 1;
        uint64_t nbytes, nrows = 0;
        if (contiguous_src && contiguous_dst) {
            if (done_bytes == total) break;
            nbytes = std::min<uint64_t>(kStageBytes, total - done_bytes);
        } else {
            if (done_rows == rows) break;
            nrows = std::min<uint64_t>(rows_per_chunk, rows - done_rows);
            nbytes = nrows * seg;
        }
        ANN_TRY(st.wait(b));
        char* stage = static_cast<char*>(st.buf[b]);
        std::atomic<bool> ok{true};
        Readers& readers = Readers::get();
        if (contiguous_src) {
            // One byte run, split into pieces of at least 1 MiB on 4 KiB boundaries.
            uint64_t const at = contiguous_dst ? file_off + done_bytes : file_off + done_rows * file_pitch;
            uint64_t const piece_min = uint64_t{1} << 20;
            int const parts = static_cast<int>(
                std::max<uint64_t>(1, std::min<uint64_t>(readers.threads(), nbytes / piece_min)));
            uint64_t const piece = ((nbytes + parts - 1) / parts + 4095) & ~uint64_t{4095};
            readers.run(parts, [&](int p) {
                uint64_t const lo = std::min<uint64_t>(nbytes, p * piece);
                uint64_t const hi = std::min<uint64_t>(nbytes, lo + piece);
                if (hi > lo && !pread_full(fd, stage + lo, hi - lo, at + lo)) ok = false;
            });
        } else {
            // One read per row, the rows split between the readers.
            int const parts = static_cast<int>(
                std::max<uint64_t>(1, std::min<uint64_t>(readers.threads(), nrows * seg >> 20)));
            uint64_t const per = (nrows + parts - 1) / parts;
            readers.run(parts, [&](int p) {
                uint64_t const r1 = std::min<uint64_t>(nrows, (p + 1) * per);
                for (uint64_t r = p * per; r < r1 && ok; ++r)
                    if (!pread_full(fd, stage + r * seg, seg, file_off + (done_rows + r) * file_pitch)) ok = false;
            });
        }
        if (!ok) return ann::fail(ANN_EIO, "loadBinaryTensor: short read for tensor '%s' in '%s'.", name, path);
        cudaError_t e;
        if (contiguous_src && contiguous_dst)
            e = cudaMemcpyAsync(dst + done_bytes, stage, nbytes, cudaMemcpyHostToDevice, s);
        else
            e = cudaMemcpy2DAsync(dst + done_rows * dst_pitch, dst_pitch, stage, seg, seg, nrows,
                                  cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess)
            return ann::fail(ANN_ECUDA, "loadBinaryTensor: copy to the device failed: %s", cudaGetErrorString(e));
        ANN_TRY(st.mark(b, s));
        done_bytes += nbytes;
        done_rows += nrows;
    }
    return ANN_OK;
}

}  // namespace

extern "C" {

int ann_sha256_file(const char* path, char hex_out[65]) {
    ANN_API_BEGIN
    if (!path || !hex_out) return ann::fail(ANN_EINVAL, "sha256File: NULL argument.");
    return sha256_of(path, hex_out);
    ANN_API_END
}

int ann_sha256_bytes(const void* data, size_t bytes, char hex_out[65]) {
    ANN_API_BEGIN
    if ((!data && bytes) || !hex_out) return ann::fail(ANN_EINVAL, "sha256: NULL argument.");
    Sha256 sha;
    sha.update(static_cast<uint8_t const*>(data), bytes);
    sha.hex(hex_out);
    return ANN_OK;
    ANN_API_END
}

int ann_load_binary_tensor(ann_stream stream, const char* path, const ann_tensor_spec* spec, size_t element_size,
                           const char* expected_sha256, void* device_out) {
    ANN_API_BEGIN
    uint64_t bytes = 0;
    ANN_TRY(validate(path, spec, element_size, expected_sha256, &bytes));
    if (!device_out) return ANN_OK;  // validation only
    Fd f(path);
    if (f.fd < 0) return ann::fail(ANN_EIO, "loadBinaryTensor: cannot open '%s'.", path);
    ::posix_fadvise(f.fd, static_cast<off_t>(spec->offset_bytes), static_cast<off_t>(bytes), POSIX_FADV_SEQUENTIAL);
    return stream_rows(ann::as_stream(stream), f.fd, path, spec->name ? spec->name : "", spec->offset_bytes, bytes,
                       bytes, 1, static_cast<char*>(device_out), bytes);
    ANN_API_END
}

int ann_load_binary_tensor_box(ann_stream stream, const char* path, const ann_tensor_spec* spec,
                               size_t element_size, const char* expected_sha256, int64_t row_begin,
                               int64_t row_count, int64_t col_begin, int64_t col_count, void* device_out,
                               int64_t out_row_pitch_bytes) {
    ANN_API_BEGIN
    uint64_t bytes = 0;
    ANN_TRY(validate(path, spec, element_size, expected_sha256, &bytes));
    if (spec->shape_rank < 1)
        return ann::fail(ANN_EINVAL, "loadBinaryTensor: a box load needs the tensor's shape (rows = shape[0]).");
    uint64_t const rows = spec->shape[0];
    uint64_t const cols = rows ? spec->count / rows : 0;
    if (row_begin < 0 || row_count <= 0 || col_begin < 0 || col_count <= 0 ||
        static_cast<uint64_t>(row_begin) + static_cast<uint64_t>(row_count) > rows ||
        static_cast<uint64_t>(col_begin) + static_cast<uint64_t>(col_count) > cols)
        return ann::fail(ANN_EINVAL,
                         "loadBinaryTensor: box rows [%lld, +%lld) x cols [%lld, +%lld) is outside the [%llu, %llu] "
                         "tensor '%s'.",
                         static_cast<long long>(row_begin), static_cast<long long>(row_count),
                         static_cast<long long>(col_begin), static_cast<long long>(col_count),
                         static_cast<unsigned long long>(rows), static_cast<unsigned long long>(cols),
                         spec->name ? spec->name : "");
    uint64_t const seg = static_cast<uint64_t>(col_count) * element_size;
    if (out_row_pitch_bytes < static_cast<int64_t>(seg) || out_row_pitch_bytes % static_cast<int64_t>(element_size))
        return ann::fail(ANN_EINVAL, "loadBinaryTensor: output row pitch %lld is below the box row (%llu bytes).",
                         static_cast<long long>(out_row_pitch_bytes), static_cast<unsigned long long>(seg));
    if (!device_out) return ANN_OK;  // validation only
    Fd f(path);
    if (f.fd < 0) return ann::fail(ANN_EIO, "loadBinaryTensor: cannot open '%s'.", path);
    uint64_t const file_pitch = cols * element_size;
    uint64_t const first = spec->offset_bytes + static_cast<uint64_t>(row_begin) * file_pitch +
                           static_cast<uint64_t>(col_begin) * element_size;
    ::posix_fadvise(f.fd, static_cast<off_t>(first), static_cast<off_t>(row_count * file_pitch),
                    POSIX_FADV_SEQUENTIAL);
    // Whole rows into a dense destination are one contiguous byte run.
    if (seg == file_pitch && out_row_pitch_bytes == static_cast<int64_t>(seg))
        return stream_rows(ann::as_stream(stream), f.fd, path, spec->name ? spec->name : "", first, seg * row_count,
                           seg * row_count, 1, static_cast<char*>(device_out), seg * row_count);
    return stream_rows(ann::as_stream(stream), f.fd, path, spec->name ? spec->name : "", first, file_pitch, seg,
                       static_cast<uint64_t>(row_count), static_cast<char*>(device_out),
                       static_cast<uint64_t>(out_row_pitch_bytes));
    ANN_API_END
}

}  // extern "C"
