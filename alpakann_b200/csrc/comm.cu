// comm.cu -- the node's NCCL communicator behind the C ABI.
//
// The head-sharded path (every rank owns H/G heads; onAcc/internal/nn/attention.hpp
// reads only head hq and KV head hq / g) re-assembles its per-rank output slabs with
// one rank-major all-gather over NVLink. NCCL is loaded with dlopen at first use
// (libnccl.so.2: in a Python process the copy PyTorch already loaded, elsewhere the
// system one), so the rest of the library does not depend on it; only its public
// types come from nccl.h. Initialisation is non-blocking and polled against a
// deadline: a rank that never joins ends in ANN_ENCCL after the deadline (the
// half-built communicator is aborted) instead of blocking for good.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "common.cuh"

namespace ann {
namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*finalize)(ncclComm_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*abort)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

NcclApi const& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (h == nullptr) return;
        auto sym = [h](auto& fn, const char* name) { fn = reinterpret_cast<std::decay_t<decltype(fn)>>(dlsym(h, name)); };
        sym(api.get_unique_id, "ncclGetUniqueId");
        sym(api.init_rank_config, "ncclCommInitRankConfig");
        sym(api.async_error, "ncclCommGetAsyncError");
        sym(api.all_gather, "ncclAllGather");
        sym(api.finalize, "ncclCommFinalize");
        sym(api.destroy, "ncclCommDestroy");
        sym(api.abort, "ncclCommAbort");
        sym(api.error_string, "ncclGetErrorString");
        api.ok = api.get_unique_id && api.init_rank_config && api.async_error && api.all_gather && api.finalize &&
                 api.destroy && api.abort && api.error_string;
    });
    return api;
}

int nccl_fail(const char* what, ncclResult_t r) {
    return fail(ANN_ENCCL, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

using Clock = std::chrono::steady_clock;

// Non-blocking communicators report ncclInProgress until a call has taken
// effect; wait for that, at most until `deadline`. An enqueued collective
// settles within microseconds, so the first 2 ms poll without sleeping (a
// sleep there would add its whole length to every step); longer waits (a
// join) back off to 100 us.
ncclResult_t settle(ncclComm_t comm, ncclResult_t r, Clock::time_point deadline) {
    auto const spin_until = Clock::now() + std::chrono::milliseconds(2);
    while (r == ncclInProgress) {
        auto const now = Clock::now();
        if (now > deadline) return ncclInProgress;
        if (now < spin_until)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(100));
        ncclResult_t state = ncclSuccess;
        ncclResult_t const q = nccl().async_error(comm, &state);
        r = q != ncclSuccess ? q : state;
    }
    return r;
}

}  // namespace
}  // namespace ann

struct ann_comm_s {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0;
    double timeout_s = 0;
};

extern "C" {

int ann_comm_unique_id(unsigned char id[ANN_COMM_ID_BYTES]) {
    ANN_API_BEGIN
    using namespace ann;
    if (id == nullptr) return fail(ANN_EINVAL, "comm unique id: null output.");
    if (!nccl().ok) return fail(ANN_ENOTSUP, "comm: libnccl.so.2 could not be loaded.");
    ncclUniqueId u;
    if (ncclResult_t r = nccl().get_unique_id(&u); r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
    static_assert(sizeof u == ANN_COMM_ID_BYTES, "NCCL unique id size");
    std::memcpy(id, &u, sizeof u);
    return ANN_OK;
    ANN_API_END
}

int ann_comm_init(ann_comm* out, int32_t nranks, int32_t rank, const unsigned char id[ANN_COMM_ID_BYTES],
                  double timeout_s) {
    ANN_API_BEGIN
    using namespace ann;
    if (out == nullptr || id == nullptr) return fail(ANN_EINVAL, "comm init: null argument.");
    *out = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks)
        return fail(ANN_EINVAL, "comm init: rank %d of %d ranks.", static_cast<int>(rank), static_cast<int>(nranks));
    if (!(timeout_s > 0)) return fail(ANN_EINVAL, "comm init: the deadline must be positive.");
    if (!nccl().ok) return fail(ANN_ENOTSUP, "comm: libnccl.so.2 could not be loaded.");
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof u);
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    ncclComm_t comm = nullptr;
    auto const deadline = Clock::now() + std::chrono::duration_cast<Clock::duration>(std::chrono::duration<double>(timeout_s));
    ncclResult_t r = nccl().init_rank_config(&comm, nranks, u, rank, &config);
    if (comm != nullptr) r = settle(comm, r, deadline);
    if (r != ncclSuccess) {
        if (comm != nullptr) nccl().abort(comm);
        if (r == ncclInProgress)
            return fail(ANN_ENCCL, "comm init: not all %d ranks joined within %.3g s.", static_cast<int>(nranks),
                        timeout_s);
        return nccl_fail("ncclCommInitRankConfig", r);
    }
    auto* c = new ann_comm_s;
    c->comm = comm;
    c->nranks = nranks;
    c->rank = rank;
    c->timeout_s = timeout_s;
    *out = c;
    return ANN_OK;
    ANN_API_END
}

int ann_comm_size(ann_comm comm, int32_t* nranks, int32_t* rank) {
    ANN_API_BEGIN
    using namespace ann;
    if (comm == nullptr) return fail(ANN_EINVAL, "comm: null communicator.");
    if (nranks) *nranks = comm->nranks;
    if (rank) *rank = comm->rank;
    return ANN_OK;
    ANN_API_END
}

int ann_comm_allgather(ann_comm comm, ann_stream stream, const void* send, void* recv, uint64_t bytes_per_rank) {
    ANN_API_BEGIN
    using namespace ann;
    if (comm == nullptr) return fail(ANN_EINVAL, "comm all-gather: null communicator.");
    if (bytes_per_rank == 0) return ANN_OK;
    if (send == nullptr || recv == nullptr) return fail(ANN_EINVAL, "comm all-gather: null buffer.");
    auto const deadline = Clock::now() + std::chrono::duration_cast<Clock::duration>(
                                             std::chrono::duration<double>(comm->timeout_s));
    ncclResult_t r = nccl().all_gather(send, recv, static_cast<size_t>(bytes_per_rank), ncclUint8, comm->comm,
                                       as_stream(stream));
    r = settle(comm->comm, r, deadline);
    if (r == ncclInProgress) return fail(ANN_ENCCL, "comm all-gather: not enqueued within %.3g s.", comm->timeout_s);
    if (r != ncclSuccess) return nccl_fail("ncclAllGather", r);
    return ANN_OK;
    ANN_API_END
}

int ann_comm_destroy(ann_comm comm) {
    ANN_API_BEGIN
    using namespace ann;
    if (comm == nullptr) return ANN_OK;
    auto const deadline = Clock::now() + std::chrono::duration_cast<Clock::duration>(
                                             std::chrono::duration<double>(comm->timeout_s));
    ncclResult_t r = settle(comm->comm, nccl().finalize(comm->comm), deadline);
    int rc = ANN_OK;
    if (r == ncclSuccess) {
        nccl().destroy(comm->comm);
    } else {  // a peer is gone or the flush did not finish: tear down without it
        nccl().abort(comm->comm);
        rc = r == ncclInProgress ? fail(ANN_ENCCL, "comm destroy: pending work did not finish within %.3g s.",
                                        comm->timeout_s)
                                 : nccl_fail("ncclCommFinalize", r);
    }
    delete comm;
    return rc;
    ANN_API_END
}

int ann_comm_abort(ann_comm comm) {
    ANN_API_BEGIN
    if (comm == nullptr) return ANN_OK;
    ann::nccl().abort(comm->comm);
    delete comm;
    return ANN_OK;
    ANN_API_END
}

}  // extern "C"
