// tma.cuh -- mbarrier, 1-D bulk-copy and tiled tensor-copy (TMA) helpers for
// sm_100a, inline PTX.
//
// Only CTA-local forms are used: a copy from global memory of THIS GPU into
// the issuing CTA's own shared memory, never to several CTAs at once.
#pragma once

#include <cstdint>

namespace ann {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Plain arrival (release semantics at CTA scope); barriers initialised with a
// count of N complete a phase after N arrivals.
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// ---- 2-CTA clusters ------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of this CTA's shared address `addr` in CTA `rank`.
__device__ __forceinline__ uint32_t map_cluster(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// Arrival on an mbarrier given by its shared::cluster address (any CTA of the
// cluster), with the default release semantics at CTA scope: the arriving
// thread's earlier writes are performed before the arrival. A cluster-scope
// release would also wait for the thread's global loads still in flight.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.release.cta.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// All threads of all CTAs of the cluster (release / acquire).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Asynchronous store of 4 / 8 bytes into shared memory of a CTA of the cluster
// (shared::cluster addresses), completing as transaction bytes on that CTA's
// mbarrier `bar_cluster`: a value reaches a peer without any barrier over the
// whole cluster.
__device__ __forceinline__ void st_async_cluster(uint32_t addr_cluster, float v, uint32_t bar_cluster) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(addr_cluster),
                 "r"(__float_as_uint(v)), "r"(bar_cluster)
                 : "memory");
}
__device__ __forceinline__ void st_async_cluster(uint32_t addr_cluster, double v, uint32_t bar_cluster) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b64 [%0], %1, [%2];" ::"r"(addr_cluster),
                 "l"(__double_as_longlong(v)), "r"(bar_cluster)
                 : "memory");
}
// try_wait with acquire semantics at cluster scope: for barriers that threads of
// another CTA of the cluster arrive on.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the phase with the given parity to complete. Returns false if it
// has not completed after `limit_ns` (the caller reports an error and stops).
// CLUSTER: acquire at cluster scope (arrivals or st.async from other CTAs).
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint64_t limit_ns = 1000000000ull) {
    auto probe = [&]() { return CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity); };
    if (probe()) return true;
    uint64_t const t0 = global_timer_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (probe()) return true;
        if (global_timer_ns() - t0 > limit_ns) return false;
    }
}

// As mbar_wait_bounded, but also gives up as soon as *abort becomes non-zero
// (another thread of the CTA has already given up). CLUSTER: the barrier's
// arrivals come from other CTAs of the cluster too (acquire at cluster scope).
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait_or_abort(uint32_t bar, uint32_t parity, volatile int* abort,
                                                   uint64_t limit_ns = 1000000000ull) {
    auto probe = [&]() { return CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity); };
    if (probe()) return true;
    uint64_t const t0 = global_timer_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (probe()) return true;
        if (*abort) return false;
        if (global_timer_ns() - t0 > limit_ns) {
            *abort = 1;
            return false;
        }
    }
}

// Bulk copy global -> own shared memory, completion signalled as transaction
// bytes on `bar`. dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Tiled tensor copy (TMA) of one box of a 4-D tensor map, global -> this
// CTA's own shared memory, completion as transaction bytes on `bar` (the full
// box, elements outside the tensor read as zero). `map` is the address of a
// __grid_constant__ CUtensorMap kernel parameter; the innermost coordinate c0
// times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* map, int c0, int c1, int c2, int c3,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}

// Tiled tensor copy (TMA) of one box from this CTA's shared memory into a
// 4-D tensor map (elements outside the tensor are not written), in the
// thread's bulk async-group. Coordinates must not be negative; c0 times the
// element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_store_4d(const void* map, int c0, int c1, int c2, int c3, uint32_t src) {
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(src)
        : "memory");
}

}  // namespace ann
