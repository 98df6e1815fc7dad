// test_dropin.cpp -- the reference's hot-path test cases (test/unit/nn/*.cpp of
// alpakaNN), written against the C++20 drop-in header alpakann_b200/onHost.hpp
// exactly as a reference user would call it: same namespaces, function names,
// template parameter and argument order. Host reference loops and known
// answers follow the reference tests; tolerance is Catch::Approx(expected)
// .epsilon(eps).margin(margin) (testHelper/test.hpp:47-54). Needs a GPU.
#include <alpakann_b200/onHost.hpp>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <limits>
#include <vector>

namespace b200 = alpaka::nn::b200;
namespace nn = alpaka::nn::onHost::nn;
namespace ops = alpaka::nn::onHost::ops;
using alpaka::nn::AttentionKvLayout;

static int g_failures = 0, g_checks = 0;

template <typename T>
static void checkValue(T actual, T expected, double eps, double margin, char const* what) {
    ++g_checks;
    double const diff = std::fabs(static_cast<double>(actual) - static_cast<double>(expected));
    if (!(diff <= margin || diff <= eps * std::fabs(static_cast<double>(expected)))) {
        if (++g_failures < 20)
            std::fprintf(stderr, "FAIL %s: %.17g vs %.17g\n", what, static_cast<double>(actual),
                         static_cast<double>(expected));
    }
}

#define REQUIRE(...)                                                              \
    do {                                                                          \
        ++g_checks;                                                               \
        if (!(__VA_ARGS__)) {                                                     \
            ++g_failures;                                                         \
            std::fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #__VA_ARGS__); \
        }                                                                         \
    } while (0)

// Device buffer + dense view, host mirror in a std::vector.
template <typename T, std::size_t R>
struct Tensor {
    std::array<int64_t, R> ext;
    std::vector<T> host;
    T* dev = nullptr;
    explicit Tensor(std::array<int64_t, R> e, T fill = T{}) : ext(e) {
        int64_t n = 1;
        for (auto x : e) n *= x;
        host.assign(static_cast<size_t>(n), fill);
        cudaMalloc(&dev, sizeof(T) * (n > 0 ? n : 1));
    }
    ~Tensor() { cudaFree(dev); }
    Tensor(Tensor const&) = delete;
    int64_t flat(std::array<int64_t, R> const& i) const {
        int64_t f = 0;
        for (std::size_t a = 0; a < R; ++a) f = f * ext[a] + i[a];
        return f;
    }
    T& operator[](std::array<int64_t, R> const& i) { return host[flat(i)]; }
    T operator[](std::array<int64_t, R> const& i) const { return host[flat(i)]; }
    void upload() { cudaMemcpy(dev, host.data(), sizeof(T) * host.size(), cudaMemcpyHostToDevice); }
    void download() { cudaMemcpy(host.data(), dev, sizeof(T) * host.size(), cudaMemcpyDeviceToHost); }
    b200::View<T, R> view() { return b200::makeView<T, R>(dev, ext); }
};

using E4 = std::array<int64_t, 4>;

// attention.cpp:24-28
template <typename T>
static void fill4D(Tensor<T, 4>& t, T base) {
    for (int64_t a = 0; a < t.ext[0]; ++a)
        for (int64_t b = 0; b < t.ext[1]; ++b)
            for (int64_t c = 0; c < t.ext[2]; ++c)
                for (int64_t d = 0; d < t.ext[3]; ++d)
                    t[{a, b, c, d}] = base + static_cast<T>(a * 101 + b * 17 + c * 7 + d * 3);
}

// attention.cpp:30-66 (scores, BTHD or BHTD)
template <typename T>
static std::vector<T> refScores(Tensor<T, 4> const& q, Tensor<T, 4> const& k, bool bhtd, int64_t Tk) {
    int64_t const B = q.ext[0], Tq = q.ext[1], H = q.ext[2], D = q.ext[3];
    std::vector<T> s(static_cast<size_t>(B * H * Tq * Tk));
    for (int64_t b = 0; b < B; ++b)
        for (int64_t h = 0; h < H; ++h)
            for (int64_t i = 0; i < Tq; ++i)
                for (int64_t j = 0; j < Tk; ++j) {
                    T sum{};
                    for (int64_t d = 0; d < D; ++d) sum += q[{b, i, h, d}] * (bhtd ? k[{b, h, j, d}] : k[{b, j, h, d}]);
                    s[((b * H + h) * Tq + i) * Tk + j] = sum;
                }
    return s;
}

// attention.cpp:115-174 (causal / plain softmax in place on [B,H,Tq,Tk])
template <typename T>
static void refSoftmax(std::vector<T>& s, int64_t rows, int64_t Tq, int64_t Tk, bool causal) {
    for (int64_t r = 0; r < rows; ++r) {
        int64_t const q = r % Tq;
        T* x = s.data() + r * Tk;
        int64_t const last = causal ? q : Tk - 1;
        T m = -std::numeric_limits<T>::infinity();
        for (int64_t j = 0; j <= last; ++j) m = std::max(m, x[j]);
        T sum{};
        for (int64_t j = 0; j < Tk; ++j) {
            if (causal && j > q) {
                x[j] = T{};
                continue;
            }
            x[j] = std::exp(x[j] - m);
            sum += x[j];
        }
        for (int64_t j = 0; j <= last; ++j) x[j] /= sum;
    }
}

// attention.cpp:68-106 (apply, BTHD or BHTD values)
template <typename T>
static std::vector<T> refApply(std::vector<T> const& p, Tensor<T, 4> const& v, bool bhtd, int64_t B, int64_t H,
                               int64_t Tq, int64_t Tk, int64_t D) {
    std::vector<T> o(static_cast<size_t>(B * Tq * H * D));
    for (int64_t b = 0; b < B; ++b)
        for (int64_t i = 0; i < Tq; ++i)
            for (int64_t h = 0; h < H; ++h)
                for (int64_t d = 0; d < D; ++d) {
                    T sum{};
                    for (int64_t j = 0; j < Tk; ++j)
                        sum += p[((b * H + h) * Tq + i) * Tk + j] * (bhtd ? v[{b, h, j, d}] : v[{b, j, h, d}]);
                    o[((b * Tq + i) * H + h) * D + d] = sum;
                }
    return o;
}

// attention.cpp:240-309 -- grouped query heads, known answers
template <typename T>
static void gqaKnownAnswers(b200::Queue& queue) {
    Tensor<T, 4> q({1, 1, 4, 2}), k({1, 1, 2, 2}), v({1, 1, 2, 2}), s({1, 4, 1, 1}), p({1, 4, 1, 1}), o({1, 1, 4, 2});
    for (int64_t h = 0; h < 4; ++h) {
        q[{0, 0, h, 0}] = static_cast<T>(h + 1);
        q[{0, 0, h, 1}] = static_cast<T>(h + 2);
    }
    k.host = {1, 2, 3, 4};
    v.host = {10, 20, 30, 40};
    q.upload(), k.upload(), v.upload();
    auto qv = q.view(), kv = k.view(), vv = v.view(), sv = s.view(), pv = p.view(), ov = o.view();
    nn::attentionScores<T>(queue, nullptr, qv, kv, sv, 2u, AttentionKvLayout::BTHD);
    nn::softmax<T>(queue, nullptr, sv, pv, 3u);
    nn::attentionApply<T>(queue, nullptr, pv, vv, ov, 2u, AttentionKvLayout::BTHD);
    queue.wait();
    s.download(), o.download();
    T const want[4] = {5, 8, 25, 32};
    for (int h = 0; h < 4; ++h) checkValue(s.host[h], want[h], 1e-5, 1e-6, "gqa scores");
    for (int h = 0; h < 4; ++h) {
        checkValue(o[{0, 0, h, 0}], static_cast<T>(h < 2 ? 10 : 30), 1e-5, 1e-6, "gqa out");
        checkValue(o[{0, 0, h, 1}], static_cast<T>(h < 2 ? 20 : 40), 1e-5, 1e-6, "gqa out");
    }
}

// attention.cpp:591-651 (prefill, causal) and :674-734 (decode, BHTD) pipelines;
// the fused kernels must give the per-op pipeline's output.
template <typename T>
static void pipeline(b200::Queue& queue, bool decode) {
    int64_t const B = 1, Tq = decode ? 1 : 4, H = 4, D = 4, Tk = decode ? 5 : 4;
    E4 const qe{B, Tq, H, D}, kvext = decode ? E4{B, H, Tk, D} : E4{B, Tk, H, D};
    Tensor<T, 4> q(qe), k(kvext), v(kvext), s({B, H, Tq, Tk}), p({B, H, Tq, Tk}), o(qe);
    fill4D<T>(q, decode ? T(0.375) : T(0.125));
    fill4D<T>(k, decode ? T(-0.0625) : T(-0.25));
    fill4D<T>(v, decode ? T(0.875) : T(0.5));
    q.upload(), k.upload(), v.upload();
    auto es = refScores<T>(q, k, decode, Tk);
    for (auto& x : es) x *= static_cast<T>(0.5);
    auto ep = es;
    refSoftmax<T>(ep, B * H * Tq, Tq, Tk, !decode);
    auto eo = refApply<T>(ep, v, decode, B, H, Tq, Tk, D);
    auto const layout = decode ? AttentionKvLayout::BHTD : AttentionKvLayout::BTHD;
    auto qv = q.view(), kv = k.view(), vv = v.view(), sv = s.view(), pv = p.view(), ov = o.view();
    nn::attentionScores<T>(queue, nullptr, qv, kv, sv, 1u, layout);
    ops::scale<T>(queue, nullptr, sv, static_cast<T>(0.5), sv);
    if (decode)
        nn::softmax<T>(queue, nullptr, sv, pv, 3u);
    else
        nn::causalSoftmax<T>(queue, nullptr, sv, pv, 3u, 2u, 3u);
    nn::attentionApply<T>(queue, nullptr, pv, vv, ov, 1u, layout);
    queue.wait();
    s.download(), p.download(), o.download();
    for (size_t i = 0; i < es.size(); ++i) checkValue(s.host[i], es[i], 1e-5, 1e-5, "pipeline scores");
    for (size_t i = 0; i < ep.size(); ++i) checkValue(p.host[i], ep[i], 1e-5, 1e-5, "pipeline probs");
    for (size_t i = 0; i < eo.size(); ++i) checkValue(o.host[i], eo[i], 1e-5, 1e-5, "pipeline out");
    // fused kernels take head dims of 64/128: pad D with zeros (scores and outputs unchanged)
    int64_t const DP = 64;
    Tensor<T, 4> q2({B, Tq, H, DP}), k2(decode ? E4{B, H, Tk, DP} : E4{B, Tk, H, DP}), v2(k2.ext), o2({B, Tq, H, DP});
    for (int64_t a = 0; a < q.ext[0]; ++a)
        for (int64_t b = 0; b < q.ext[1]; ++b)
            for (int64_t c = 0; c < q.ext[2]; ++c)
                for (int64_t d = 0; d < D; ++d) q2[{a, b, c, d}] = q[{a, b, c, d}];
    for (int64_t a = 0; a < k.ext[0]; ++a)
        for (int64_t b = 0; b < k.ext[1]; ++b)
            for (int64_t c = 0; c < k.ext[2]; ++c)
                for (int64_t d = 0; d < D; ++d) k2[{a, b, c, d}] = k[{a, b, c, d}], v2[{a, b, c, d}] = v[{a, b, c, d}];
    q2.upload(), k2.upload(), v2.upload();
    auto q2v = q2.view(), k2v = k2.view(), v2v = v2.view(), o2v = o2.view();
    if (decode)
        nn::attentionDecode<T>(queue, nullptr, q2v, k2v, v2v, o2v, static_cast<T>(0.5), 1u, layout);
    else
        nn::attentionPrefill<T>(queue, nullptr, q2v, k2v, v2v, o2v, static_cast<T>(0.5), 1u, layout, true);
    queue.wait();
    o2.download();
    for (int64_t i = 0; i < Tq; ++i)
        for (int64_t h = 0; h < H; ++h)
            for (int64_t d = 0; d < D; ++d)
                checkValue(o2[{0, i, h, d}], eo[(i * H + h) * D + d], 1e-5, 1e-5, "fused out");
}

// softmax.cpp:88-114 -- large logits, causal zeros, rows sum to 1
template <typename T>
static void softmaxStability(b200::Queue& queue) {
    Tensor<T, 4> in({1, 1, 2, 3}), out({1, 1, 2, 3});
    in.host = {1000, 1001, 999, -1, 0, 1};
    in.upload();
    auto iv = in.view(), ov = out.view();
    nn::causalSoftmax<T>(queue, nullptr, iv, ov, 3u, 2u, 3u);
    queue.wait();
    out.download();
    REQUIRE(out.host[1] == T{});
    REQUIRE(out.host[2] == T{});
    checkValue(out.host[0], T{1}, 1e-5, 1e-6, "row 0 sum");
    checkValue(out.host[3] + out.host[4] + out.host[5], T{1}, 1e-5, 1e-6, "row 1 sum");
}

// rope.cpp:20-82 and attention.cpp:852-975 (qkvProjection + ropeInPlace on flat buffers)
template <typename T>
static void qkvRope(b200::Queue& queue) {
    int64_t const tokens = 3, hidden = 4, pairs = 2;
    Tensor<T, 2> x({tokens, hidden}), wq({hidden, hidden}), wk({hidden, hidden}), wv({hidden, hidden});
    Tensor<T, 2> cosT({tokens, pairs}), sinT({tokens, pairs});
    for (int64_t r = 0; r < tokens; ++r)
        for (int64_t c = 0; c < hidden; ++c)
            x[{r, c}] = static_cast<T>(-0.25) + static_cast<T>(r * 13 + c * 3) * static_cast<T>(0.05);
    for (int64_t r = 0; r < hidden; ++r)
        for (int64_t c = 0; c < hidden; ++c) {
            T const f = static_cast<T>(r * hidden + c);
            wq[{r, c}] = static_cast<T>(-0.1) + f * static_cast<T>(0.01);
            wk[{r, c}] = static_cast<T>(0.2) - f * static_cast<T>(0.007);
            wv[{r, c}] = static_cast<T>(-0.05) + f * static_cast<T>(0.009);
        }
    for (int64_t pos = 0; pos < tokens; ++pos)
        for (int64_t pr = 0; pr < pairs; ++pr) {
            T const ang = static_cast<T>(pos + 1) * static_cast<T>(0.25) * static_cast<T>(pr + 1);
            cosT[{pos, pr}] = std::cos(ang);
            sinT[{pos, pr}] = std::sin(ang);
        }
    auto proj = [&](Tensor<T, 2>& w) {
        std::vector<T> e(static_cast<size_t>(tokens * hidden));
        for (int64_t r = 0; r < tokens; ++r)
            for (int64_t c = 0; c < hidden; ++c) {
                T sum{};
                for (int64_t i = 0; i < hidden; ++i) sum += x[{r, i}] * w[{i, c}];
                e[r * hidden + c] = sum;
            }
        return e;
    };
    auto rot = [&](std::vector<T> e) {
        for (int64_t t = 0; t < tokens; ++t)
            for (int64_t pr = 0; pr < pairs; ++pr) {
                T const c = cosT[{t, pr}], s = sinT[{t, pr}];
                T const x0 = e[t * hidden + 2 * pr], x1 = e[t * hidden + 2 * pr + 1];
                e[t * hidden + 2 * pr] = x0 * c - x1 * s;
                e[t * hidden + 2 * pr + 1] = x0 * s + x1 * c;
            }
        return e;
    };
    auto eq = rot(proj(wq)), ek = rot(proj(wk)), ev = proj(wv);
    for (auto* t : {&x, &wq, &wk, &wv, &cosT, &sinT}) t->upload();
    Tensor<T, 1> qf({tokens * hidden}), kf({tokens * hidden}), vf({tokens * hidden});
    auto q2 = b200::makeView<T, 2>(qf.dev, {tokens, hidden}), k2 = b200::makeView<T, 2>(kf.dev, {tokens, hidden}),
         v2 = b200::makeView<T, 2>(vf.dev, {tokens, hidden});
    auto xv = x.view(), wqv = wq.view(), wkv = wk.view(), wvv = wv.view();
    nn::qkvProjection<T>(queue, xv, wqv, wkv, wvv, q2, k2, v2);
    auto q4 = b200::makeView<T, 4>(qf.dev, {1, tokens, 1, hidden}), k4 = b200::makeView<T, 4>(kf.dev, {1, tokens, 1, hidden});
    auto cv = cosT.view(), sv = sinT.view();
    nn::ropeInPlace<T>(queue, nullptr, q4, k4, cv, sv);
    queue.wait();
    qf.download(), kf.download(), vf.download();
    for (size_t i = 0; i < eq.size(); ++i) {
        checkValue(qf.host[i], eq[i], 1e-5, 1e-5, "q");
        checkValue(kf.host[i], ek[i], 1e-5, 1e-5, "k");
        checkValue(vf.host[i], ev[i], 1e-5, 1e-5, "v");
    }
}

// rms_norm.cpp:18-48
template <typename T>
static void rmsNorm(b200::Queue& queue) {
    Tensor<T, 2> in({2, 4}), out({2, 4});
    Tensor<T, 1> w({4});
    for (int64_t r = 0; r < 2; ++r)
        for (int64_t c = 0; c < 4; ++c) in[{r, c}] = static_cast<T>(r * 4 + c + 1);
    for (int64_t i = 0; i < 4; ++i) w[{i}] = static_cast<T>(0.5) + static_cast<T>(i);
    in.upload(), w.upload();
    auto iv = in.view(), wv = w.view(), ov = out.view();
    nn::rmsNorm<T>(queue, nullptr, iv, wv, ov, static_cast<T>(1.0e-5));
    queue.wait();
    out.download();
    for (int64_t r = 0; r < 2; ++r) {
        T ss{};
        for (int64_t c = 0; c < 4; ++c) ss += in[{r, c}] * in[{r, c}];
        T const inv = T{1} / std::sqrt(ss / T{4} + static_cast<T>(1.0e-5));
        for (int64_t c = 0; c < 4; ++c) checkValue(out[{r, c}], in[{r, c}] * inv * w[{c}], 1e-5, 1e-6, "rmsNorm");
    }
}

// embedding.cpp:20-170 -- gather, non-contiguous subview, validation throws
template <typename T>
static void embedding(b200::Queue& queue) {
    Tensor<T, 2> storage({3, 5});
    for (int64_t r = 0; r < 3; ++r)
        for (int64_t c = 0; c < 5; ++c) storage[{r, c}] = static_cast<T>(r * 10 + c);
    storage.upload();
    Tensor<uint32_t, 1> ids({4});
    ids.host = {2, 0, 1, 2};
    ids.upload();
    Tensor<T, 2> out({4, 2});
    auto table = b200::subView<T, 2>(storage.view(), {0, 2}, {3, 2});
    auto idv = ids.view(), ov = out.view();
    nn::embeddingLookup<T>(queue, nullptr, idv, table, ov);
    queue.wait();
    out.download();
    for (int64_t t = 0; t < 4; ++t)
        for (int64_t c = 0; c < 2; ++c) REQUIRE(out[{t, c}] == storage[{static_cast<int64_t>(ids.host[t]), 2 + c}]);
    Tensor<T, 2> wrongRows({3, 2}), wrongCols({4, 3});
    Tensor<T, 3> wrongRank({4, 2, 1});
    bool threw = false;
    try {
        auto v = wrongRows.view();
        nn::embeddingLookup<T>(queue, nullptr, idv, table, v);
    } catch (std::invalid_argument const&) {
        threw = true;
    }
    REQUIRE(threw);
    threw = false;
    try {
        auto v = wrongCols.view();
        nn::embeddingLookup<T>(queue, nullptr, idv, table, v);
    } catch (std::invalid_argument const&) {
        threw = true;
    }
    REQUIRE(threw);
    threw = false;
    try {
        auto v = wrongRank.view();
        nn::embeddingLookup<T>(queue, nullptr, idv, table, v);
    } catch (std::invalid_argument const&) {
        threw = true;
    }
    REQUIRE(threw);
    threw = false;
    try {
        auto qv = out.view();
        nn::attentionScores<T>(queue, nullptr, qv, qv, qv, 0u);
    } catch (std::invalid_argument const&) {
        threw = true;
    }
    REQUIRE(threw);
}

// The head-sharded decode step through a 1-rank communicator: RoPE, decode,
// all-gather and re-assembly must give exactly the plain RoPE + decode result.
template <typename T>
static void headShardedOneRank(b200::Queue& queue) {
    int64_t const B = 2, H = 4, Tk = 40, D = 64;
    Tensor<T, 4> q({B, 1, H, D}), kn({B, 1, H, D}), q2({B, 1, H, D}), kn2({B, 1, H, D});
    Tensor<T, 4> kc({B, H, Tk, D}), vc({B, H, Tk, D}), local({B, 1, H, D}), out({B, 1, H, D}), ref({B, 1, H, D});
    Tensor<T, 5> gathered({1, B, 1, H, D});
    Tensor<T, 2> cosT({Tk + 1, D / 2}), sinT({Tk + 1, D / 2});
    fill4D<T>(q, T(0.25)), fill4D<T>(kn, T(-0.5)), fill4D<T>(kc, T(0.125)), fill4D<T>(vc, T(0.75));
    q2.host = q.host, kn2.host = kn.host;
    for (int64_t p = 0; p <= Tk; ++p)
        for (int64_t i = 0; i < D / 2; ++i) {
            double const a = static_cast<double>(p) * std::pow(10000.0, -2.0 * static_cast<double>(i) / D);
            cosT[{p, i}] = static_cast<T>(std::cos(a)), sinT[{p, i}] = static_cast<T>(std::sin(a));
        }
    for (auto* t : {&q, &kn, &q2, &kn2, &kc, &vc}) t->upload();
    cosT.upload(), sinT.upload();
    auto qv = q.view(), knv = kn.view(), q2v = q2.view(), kn2v = kn2.view(), kcv = kc.view(), vcv = vc.view();
    auto lv = local.view(), ov = out.view(), rv = ref.view(), cv = cosT.view(), sv = sinT.view();
    auto gv = gathered.view();
    T const scale = static_cast<T>(0.125);
    {
        b200::Comm comm(1, 0, b200::Comm::uniqueId(), 30.0);
        REQUIRE(comm.size() == 1);
        b200::headShardedDecode<T>(queue, comm, qv, knv, cv, sv, static_cast<uint32_t>(Tk), kcv, vcv, lv, gv, ov,
                                   scale);
        queue.wait();
    }
    nn::ropeInPlace<T>(queue, nullptr, q2v, kn2v, cv, sv, alpaka::nn::RopeLayout::BTHD, static_cast<uint32_t>(Tk));
    nn::attentionDecode<T>(queue, nullptr, q2v, kcv, vcv, rv, scale, 1u, AttentionKvLayout::BHTD);
    queue.wait();
    out.download(), ref.download();
    REQUIRE(out.host == ref.host);
}

// core/binary.cpp:70-121 (roundtrip behind a 64-byte poison prefix, digest
// checked) and :182-235 (every rejected layout, and the exception type).
template <typename T>
static void binaryTensor(b200::Queue& queue) {
    namespace onHost = alpaka::nn::onHost;
    auto const path = (std::filesystem::temp_directory_path() / "alpakann_b200_dropin_binary.bin").string();
    std::vector<T> values(6);
    for (std::size_t i = 0; i < values.size(); ++i) values[i] = static_cast<T>(i) * T(0.5) - T(1.25);
    {
        std::vector<unsigned char> bytes(64, 0xab);
        bytes.resize(64 + values.size() * sizeof(T));
        std::memcpy(bytes.data() + 64, values.data(), values.size() * sizeof(T));
        std::ofstream f(path, std::ios::binary | std::ios::trunc);
        f.write(reinterpret_cast<char const*>(bytes.data()), static_cast<std::streamsize>(bytes.size()));
    }
    onHost::TensorSpec const spec{"t", 64u, 6u, {2u, 3u}};
    auto const sha = onHost::sha256File(path);
    REQUIRE(sha.size() == 64u);
    auto buffer = onHost::loadBinaryTensor<T>(queue, path, spec, sha);
    queue.wait();
    std::vector<T> back(6);
    cudaMemcpy(back.data(), buffer.data(), sizeof(T) * back.size(), cudaMemcpyDeviceToHost);
    REQUIRE(back == values);
    REQUIRE(buffer.getExtents()[0] == 6);

    auto throwsAs = [&](auto fn, bool invalidArgument) {
        bool ok = false;
        try {
            fn();
        } catch (std::invalid_argument const&) {
            ok = invalidArgument;
        } catch (std::runtime_error const&) {
            ok = !invalidArgument;
        }
        REQUIRE(ok);
    };
    auto mk = [](std::size_t off, std::size_t count, std::vector<std::size_t> shape = {}) {
        return onHost::TensorSpec{"spec", off, count, std::move(shape)};
    };
    throwsAs([&] { onHost::loadBinaryTensor<T>(queue, path, mk(8u, 4u)); }, true);
    throwsAs([&] { onHost::loadBinaryTensor<T>(queue, path, mk(0u, 6u, {2u, 4u})); }, true);
    throwsAs([&] { onHost::loadBinaryTensor<T>(queue, path, mk(0u, 1000u)); }, true);
    throwsAs([&] { onHost::loadBinaryTensor<T>(queue, path, mk(0u, std::numeric_limits<std::size_t>::max() / sizeof(T) + 1u)); }, true);
    throwsAs([&] { onHost::loadBinaryTensor<T>(queue, path, mk(0u, 0u)); }, true);
    throwsAs([&] { onHost::loadBinaryTensor<T>(queue, path, mk(0u, 4u), std::string(64u, '0')); }, false);
    throwsAs([&] { onHost::loadBinaryTensor<T>(queue, path + ".missing", mk(0u, 4u)); }, false);
    std::filesystem::remove(path);
}

// ops/elementwise.cpp:31-130: the elementwise chain on [2,4], biasAdd, cast,
// and the activations on padded views (row pitch 8).
template <typename T>
static void elementwise(b200::Queue& queue) {
    Tensor<T, 2> a({2, 4}), b({2, 4}), out({2, 4});
    T v = T(-3);
    for (auto& x : a.host) x = v, v += T(0.5);
    for (std::size_t i = 0; i < b.host.size(); ++i) b.host[i] = a.host[i] + T(1);
    a.upload(), b.upload();
    auto av = a.view(), bv = b.view(), ov = out.view();
    ops::fill(queue, nullptr, ov, T(2));
    ops::copy(queue, nullptr, av, ov);
    ops::add<T>(queue, nullptr, av, bv, ov);
    queue.wait(), out.download();
    for (std::size_t i = 0; i < 8; ++i) checkValue(out.host[i], T(a.host[i] + b.host[i]), 1e-5, 1e-6, "add");
    ops::sub<T>(queue, nullptr, bv, av, ov);
    ops::mul<T>(queue, nullptr, av, bv, ov);
    ops::div<T>(queue, nullptr, bv, av, ov);
    ops::scale<T>(queue, nullptr, av, T(3), ov);
    ops::axpy<T>(queue, nullptr, T(2), av, bv, ov);
    queue.wait(), out.download();
    for (std::size_t i = 0; i < 8; ++i) checkValue(out.host[i], T(T(2) * a.host[i] + b.host[i]), 1e-5, 1e-6, "axpy");
    Tensor<T, 1> bias({4});
    for (int i = 0; i < 4; ++i) bias.host[static_cast<std::size_t>(i)] = static_cast<T>(i);
    bias.upload();
    auto biv = bias.view();
    ops::biasAdd(queue, nullptr, av, biv, ov);
    queue.wait(), out.download();
    for (std::size_t i = 0; i < 8; ++i) checkValue(out.host[i], T(a.host[i] + bias.host[i % 4]), 1e-5, 1e-6, "bias");
    int* idev = nullptr;
    cudaMalloc(&idev, 8 * sizeof(int));
    auto iv = b200::makeView<int, 2>(idev, {2, 4});
    ops::cast<int>(queue, nullptr, av, iv);
    queue.wait();
    int ih[8];
    cudaMemcpy(ih, idev, sizeof(ih), cudaMemcpyDeviceToHost);
    for (std::size_t i = 0; i < 8; ++i) REQUIRE(ih[i] == static_cast<int>(a.host[i]));
    cudaFree(idev);
    // padded views: 24 elements, [2,4] with row pitch 8 elements
    Tensor<T, 1> pin({24}), pout({24});
    for (int r = 0; r < 2; ++r)
        for (int c = 0; c < 4; ++c) pin.host[static_cast<std::size_t>(r * 8 + c)] = a.host[static_cast<std::size_t>(r * 4 + c)];
    pin.upload(), pout.upload();
    b200::View<T, 2> vin{pin.dev, {2, 4}, {8 * int64_t(sizeof(T)), int64_t(sizeof(T))}};
    b200::View<T, 2> vout{pout.dev, {2, 4}, {8 * int64_t(sizeof(T)), int64_t(sizeof(T))}};
    ops::exp<T>(queue, nullptr, vin, vout);
    ops::sqrt<T>(queue, nullptr, vout, vout);
    ops::rsqrt<T>(queue, nullptr, vout, vout);
    ops::relu<T>(queue, nullptr, vin, vout);
    ops::sigmoid<T>(queue, nullptr, vin, vout);
    ops::silu<T>(queue, nullptr, vin, vout);
    ops::gelu<T>(queue, nullptr, vin, vout);
    ops::swiglu<T>(queue, nullptr, vin, vin, vout);
    queue.wait(), pout.download();
    double const eps = std::is_same_v<T, float> ? 1e-5 : 1e-9;
    for (int r = 0; r < 2; ++r)
        for (int c = 0; c < 4; ++c) {
            T const x = a.host[static_cast<std::size_t>(r * 4 + c)];
            T const sig = T(1) / (T(1) + std::exp(-x));
            checkValue(pout.host[static_cast<std::size_t>(r * 8 + c)], T(x * sig * x), eps, eps, "swiglu padded");
            REQUIRE(pout.host[static_cast<std::size_t>(r * 8 + c + 4)] == T(0));
        }
}

// ops/reduction.cpp:33-124
template <typename T>
static void reductions(b200::Queue& queue) {
    Tensor<T, 3> in({2, 3, 4}), out({2, 3, 1});
    for (std::size_t i = 0; i < in.host.size(); ++i) in.host[i] = static_cast<T>(i + 1);
    in.upload();
    auto iv = in.view(), ov = out.view();
    REQUIRE((ops::makeReducedExtents(iv.getExtents(), 2u) == std::array<int64_t, 3>{2, 3, 1}));
    double const eps = std::is_same_v<T, float> ? 1e-5 : 1e-12;
    ops::reduceSum<T>(queue, nullptr, iv, ov, 2u);
    queue.wait(), out.download();
    for (int r = 0; r < 6; ++r) {
        T sum{};
        for (int k = 0; k < 4; ++k) sum += in.host[static_cast<std::size_t>(r * 4 + k)];
        checkValue(out.host[static_cast<std::size_t>(r)], sum, eps, eps, "reduceSum");
    }
    ops::reduceMean<T>(queue, nullptr, iv, ov, 2u);
    ops::reduceMax<T>(queue, nullptr, iv, ov, 2u);
    queue.wait(), out.download();
    for (int r = 0; r < 6; ++r) REQUIRE(out.host[static_cast<std::size_t>(r)] == in.host[static_cast<std::size_t>(r * 4 + 3)]);
    ops::reduceSumSquares<T>(queue, nullptr, iv, ov, 2u);
    queue.wait(), out.download();
    for (int r = 0; r < 6; ++r) {
        T sum{};
        for (int k = 0; k < 4; ++k) sum += in.host[static_cast<std::size_t>(r * 4 + k)] * in.host[static_cast<std::size_t>(r * 4 + k)];
        checkValue(out.host[static_cast<std::size_t>(r)], sum, eps, eps, "reduceSumSquares");
    }
    Tensor<T, 3> dotOut({2, 1, 4});
    auto dv = dotOut.view();
    ops::dot<T>(queue, nullptr, iv, iv, dv, 1u);
    queue.wait(), dotOut.download();
    for (int b = 0; b < 2; ++b)
        for (int k = 0; k < 4; ++k) {
            T sum{};
            for (int j = 0; j < 3; ++j) {
                T const x = in.host[static_cast<std::size_t>(b * 12 + j * 4 + k)];
                sum += x * x;
            }
            checkValue(dotOut.host[static_cast<std::size_t>(b * 4 + k)], sum, eps, eps, "dot");
        }
    bool threw = false;
    try {
        ops::reduceSum<T>(queue, nullptr, iv, iv, 2u);
    } catch (std::invalid_argument const&) {
        threw = true;
    }
    REQUIRE(threw);
}

// nn/mlp.cpp:20-68 and nn/mlp_forward.cpp:60-216
template <typename T>
static void mlpCases(b200::Queue& queue) {
    Tensor<T, 2> x({1, 4}), wg({4, 6}), wu({4, 6}), wd({6, 4}), out({1, 4});
    for (int k = 0; k < 4; ++k) x.host[static_cast<std::size_t>(k)] = static_cast<T>(k + 1);
    for (int k = 0; k < 4; ++k)
        for (int c = 0; c < 6; ++c) {
            wg[{k, c}] = T(0.05) * static_cast<T>(k + c + 1);
            wu[{k, c}] = T(0.04) * static_cast<T>(k + c + 1);
        }
    for (int k = 0; k < 6; ++k)
        for (int c = 0; c < 4; ++c) wd[{k, c}] = T(0.03) * static_cast<T>(k + c + 1);
    for (auto* t : {&x, &wg, &wu, &wd}) t->upload();
    auto xv = x.view(), gv = wg.view(), uv = wu.view(), dv = wd.view(), ov = out.view();
    nn::mlp<T>(queue, nullptr, xv, gv, uv, dv, ov);
    queue.wait(), out.download();
    T hidden[6];
    for (int c = 0; c < 6; ++c) {
        T a{}, b{};
        for (int k = 0; k < 4; ++k) a += x.host[static_cast<std::size_t>(k)] * wg[{k, c}], b += x.host[static_cast<std::size_t>(k)] * wu[{k, c}];
        hidden[c] = a / (T(1) + std::exp(-a)) * b;
    }
    for (int c = 0; c < 4; ++c) {
        T e{};
        for (int k = 0; k < 6; ++k) e += hidden[k] * wd[{k, c}];
        checkValue(out.host[static_cast<std::size_t>(c)], e, 1e-5, 1e-6, "mlp");
    }

    auto fillDet = [](auto& t, T scale, T shift) {
        for (std::size_t i = 0; i < t.host.size(); ++i) t.host[i] = scale * static_cast<T>(i + 1) + shift;
        t.upload();
    };
    auto silu = [](T v) { return v / (T(1) + std::exp(-v)); };
    // three layers, silu hidden, none last (mlp_forward.cpp:112-182)
    Tensor<T, 2> in({2, 3}), w0({3, 5}), w1({5, 4}), w2({4, 2}), res({2, 2});
    Tensor<T, 1> b0({5}), b1({4}), b2({2});
    fillDet(in, T(0.2), T(-0.3)), fillDet(w0, T(0.09), T(-0.2)), fillDet(w1, T(0.07), T(-0.1));
    fillDet(w2, T(0.05), T(-0.05)), fillDet(b0, T(0.03), T(0.01)), fillDet(b1, T(0.02), T(-0.01));
    fillDet(b2, T(0.01), T(0.02));
    using W = nn::WeightView<b200::View<T, 2>>;
    using B = nn::BiasView<b200::View<T, 1>>;
    std::array<W, 3> ws{W{w0.view()}, W{w1.view()}, W{w2.view()}};
    std::array<B, 3> bs{B{b0.view()}, B{b1.view()}, B{b2.view()}};
    auto inv = in.view(), rv = res.view();
    nn::mlpForward<T>(queue, nullptr, inv, ws, bs, nn::Activation::silu, nn::Activation::none, rv);
    queue.wait(), res.download();
    for (int r = 0; r < 2; ++r) {
        T l0[5], l1[4];
        for (int c = 0; c < 5; ++c) {
            T v = b0.host[static_cast<std::size_t>(c)];
            for (int k = 0; k < 3; ++k) v += in[{r, k}] * w0[{k, c}];
            l0[c] = silu(v);
        }
        for (int c = 0; c < 4; ++c) {
            T v = b1.host[static_cast<std::size_t>(c)];
            for (int k = 0; k < 5; ++k) v += l0[k] * w1[{k, c}];
            l1[c] = silu(v);
        }
        for (int c = 0; c < 2; ++c) {
            T v = b2.host[static_cast<std::size_t>(c)];
            for (int k = 0; k < 4; ++k) v += l1[k] * w2[{k, c}];
            checkValue(res[{r, c}], v, 1e-5, 1e-6, "mlpForward 3 layers");
        }
    }
    // decodeLatent (mlp_forward.cpp:184-216)
    Tensor<T, 2> lat({1, 3}), wl({3, 5}), lo({1, 5});
    fillDet(lat, T(0.4), T(-0.6)), fillDet(wl, T(0.08), T(-0.3));
    auto lav = lat.view(), wlv = wl.view(), lov = lo.view();
    nn::decodeLatent<T>(queue, nullptr, lav, wlv, lov);
    queue.wait(), lo.download();
    for (int c = 0; c < 5; ++c) {
        T e{};
        for (int k = 0; k < 3; ++k) e += lat.host[static_cast<std::size_t>(k)] * wl[{k, c}];
        checkValue(lo.host[static_cast<std::size_t>(c)], e, 1e-5, 1e-6, "decodeLatent");
    }
    // maskedSoftmax with a -inf mask: masked entries 0, the rest sum to 1
    Tensor<T, 2> sIn({2, 5}), sMask({2, 5}), sOut({2, 5});
    for (int i = 0; i < 10; ++i) {
        sIn.host[static_cast<std::size_t>(i)] = static_cast<T>(i % 5);
        sMask.host[static_cast<std::size_t>(i)] = (i % 5 >= 3) ? -std::numeric_limits<T>::infinity() : T(0);
    }
    sIn.upload(), sMask.upload();
    auto siv = sIn.view(), smv = sMask.view(), sov = sOut.view();
    nn::maskedSoftmax<T>(queue, nullptr, siv, smv, sov, 1u);
    queue.wait(), sOut.download();
    T const z = std::exp(T(-2)) + std::exp(T(-1)) + T(1);
    for (int r = 0; r < 2; ++r)
        for (int c = 0; c < 5; ++c)
            checkValue(sOut[{r, c}], c >= 3 ? T(0) : T(std::exp(static_cast<T>(c - 2)) / z), 1e-5, 1e-7, "maskedSoftmax");
}

template <typename T>
static void all(b200::Queue& queue) {
    gqaKnownAnswers<T>(queue);
    pipeline<T>(queue, false);
    pipeline<T>(queue, true);
    softmaxStability<T>(queue);
    qkvRope<T>(queue);
    rmsNorm<T>(queue);
    embedding<T>(queue);
    headShardedOneRank<T>(queue);
    binaryTensor<T>(queue);
    elementwise<T>(queue);
    reductions<T>(queue);
    mlpCases<T>(queue);
}

int main() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        std::fprintf(stderr, "no CUDA device\n");
        return 2;
    }
    b200::Queue queue(0);
    all<float>(queue);
    all<double>(queue);
    std::printf("%d checks, %d failures\n", g_checks, g_failures);
    return g_failures == 0 ? 0 : 1;
}
