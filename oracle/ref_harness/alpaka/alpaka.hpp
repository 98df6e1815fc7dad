// alpaka/alpaka.hpp -- a host-only STAND-IN for the few parts of the alpaka3
// API that alpakaNN's device kernels (include/alpaka/nn/onAcc/internal/nn/*.hpp)
// use, so that those kernel sources compile UNMODIFIED with g++ and run on the
// host as the parity reference of the CPU oracle.
//
// TEST INFRASTRUCTURE ONLY (oracle/_ref). This is not alpaka and contains none
// of its code: it provides just the names and semantics the kernels call,
// written for this harness --
//   ALPAKA_FN_ACC, ALPAKA_TYPEOF, alpaka::unused,
//   alpaka::Vec (index vector: brace construction, operator[], static dim()),
//   alpaka::IdxRange{extents} and alpaka::onAcc::makeIdxMap(acc,
//     worker::threadsInGrid, range): every index of the range, row-major,
//     one after the other (a single host thread is the whole "grid"),
//   alpaka::math::{exp, rsqrt, max} on the host: std::exp, 1 / std::sqrt,
//     std::fmax (the forms alpaka's CPU back end uses for float and double).
// Views are supplied by the harness (ref_kernels.cpp): any type with
// getExtents() returning an alpaka::Vec and operator[](alpaka::Vec) -> T&.
#pragma once

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdint>
#include <type_traits>

#define ALPAKA_FN_ACC
#define ALPAKA_TYPEOF(...) std::remove_cvref_t<decltype(__VA_ARGS__)>

namespace alpaka {

template <typename... T>
constexpr void unused(T const&...) {}

template <typename T_Idx, uint32_t T_dim>
struct Vec {
    std::array<T_Idx, T_dim> v{};

    constexpr Vec() = default;
    template <typename... T>
        requires(sizeof...(T) == T_dim && (std::is_integral_v<T> && ...))
    constexpr Vec(T... xs) : v{static_cast<T_Idx>(xs)...} {}

    static constexpr uint32_t dim() { return T_dim; }
    constexpr T_Idx& operator[](std::integral auto i) { return v[static_cast<std::size_t>(i)]; }
    constexpr T_Idx const& operator[](std::integral auto i) const { return v[static_cast<std::size_t>(i)]; }
};
template <typename... T>
Vec(T...) -> Vec<std::common_type_t<T...>, sizeof...(T)>;

template <typename T_Vec>
struct IdxRange {
    T_Vec extents;
};
template <typename T_Vec>
IdxRange(T_Vec) -> IdxRange<T_Vec>;

namespace onAcc {
namespace worker {
struct ThreadsInGrid {};
inline constexpr ThreadsInGrid threadsInGrid{};
}  // namespace worker

// Row-major walk over every index of a range (last axis fastest).
template <typename T_Vec>
struct IdxWalk {
    T_Vec extents;
    struct iterator {
        T_Vec idx;
        T_Vec extents;
        bool done;
        T_Vec const& operator*() const { return idx; }
        iterator& operator++() {
            for (int a = static_cast<int>(T_Vec::dim()) - 1; a >= 0; --a) {
                if (++idx[a] < extents[a]) return *this;
                idx[a] = 0;
            }
            done = true;
            return *this;
        }
        bool operator!=(iterator const& o) const { return done != o.done; }
    };
    iterator begin() const {
        bool empty = false;
        for (uint32_t a = 0; a < T_Vec::dim(); ++a) empty = empty || extents[a] == 0;
        return iterator{T_Vec{}, extents, empty};
    }
    iterator end() const { return iterator{T_Vec{}, extents, true}; }
};

template <typename T_Acc, typename T_Vec>
IdxWalk<T_Vec> makeIdxMap(T_Acc const&, worker::ThreadsInGrid, IdxRange<T_Vec> const& range) {
    return IdxWalk<T_Vec>{range.extents};
}
}  // namespace onAcc

namespace math {
template <typename T>
T exp(T x) {
    return std::exp(x);
}
template <typename T>
T rsqrt(T x) {
    return static_cast<T>(1) / std::sqrt(x);
}
template <typename T>
T max(T a, T b) {
    if constexpr (std::is_floating_point_v<T>)
        return std::fmax(a, b);
    else
        return std::max(a, b);
}
}  // namespace math

}  // namespace alpaka
