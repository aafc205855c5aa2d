// Data-parallel gradient averaging for C / C++ callers without torch: NCCL is
// loaded at run time (libnccl.so.2 — the copy already in the process when there is
// one), so the library has no link-time NCCL dependency (nccl.h supplies only the
// types). One process per GPU; the flat gradient buffer is all-reduced once per
// step (sum, or average over ranks).
//
// Failure handling: the communicator is created non-blocking, so no NCCL call
// blocks the host. Set-up and bsml_nccl_sync poll against a host deadline; when a
// peer has left (it never joins the collective) or NCCL reports an asynchronous
// error, the communicator is aborted — which ends its kernels still waiting on
// the GPU — and the call returns an error instead of hanging.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "common.cuh"
#include "nccl_dl.h"

namespace bsml {

namespace {

using fn_get_version = ncclResult_t (*)(int*);
using fn_get_unique_id = ncclResult_t (*)(ncclUniqueId*);
using fn_comm_init_rank_config = ncclResult_t (*)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
using fn_comm_destroy = ncclResult_t (*)(ncclComm_t);
using fn_comm_abort = ncclResult_t (*)(ncclComm_t);
using fn_get_async_error = ncclResult_t (*)(ncclComm_t, ncclResult_t*);
using fn_all_reduce = ncclResult_t (*)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                       cudaStream_t);
using fn_error_string = const char* (*)(ncclResult_t);

// non-blocking communicators, ncclCommGetAsyncError / ncclCommAbort on them and
// ncclAvg (2.10) all hold from this release on
constexpr int kMinVersion = 21400;

struct Nccl {
    void* h = nullptr;
    int version = 0;
    fn_get_unique_id get_unique_id = nullptr;
    fn_comm_init_rank_config init_config = nullptr;
    fn_comm_destroy comm_destroy = nullptr;
    fn_comm_abort comm_abort = nullptr;
    fn_get_async_error async_error = nullptr;
    fn_all_reduce all_reduce = nullptr;
    fn_error_string error_string = nullptr;
};

const Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    static std::string err;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char* e = dlerror();
            err = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown");
            return;
        }
        n.h = h;
        auto get_version = reinterpret_cast<fn_get_version>(dlsym(h, "ncclGetVersion"));
        n.get_unique_id = reinterpret_cast<fn_get_unique_id>(dlsym(h, "ncclGetUniqueId"));
        n.init_config = reinterpret_cast<fn_comm_init_rank_config>(dlsym(h, "ncclCommInitRankConfig"));
        n.comm_destroy = reinterpret_cast<fn_comm_destroy>(dlsym(h, "ncclCommDestroy"));
        n.comm_abort = reinterpret_cast<fn_comm_abort>(dlsym(h, "ncclCommAbort"));
        n.async_error = reinterpret_cast<fn_get_async_error>(dlsym(h, "ncclCommGetAsyncError"));
        n.all_reduce = reinterpret_cast<fn_all_reduce>(dlsym(h, "ncclAllReduce"));
        n.error_string = reinterpret_cast<fn_error_string>(dlsym(h, "ncclGetErrorString"));
        if (!get_version || get_version(&n.version) != ncclSuccess) {
            err = "libnccl.so.2 does not report its version (NCCL 2.14 or later is required)";
            return;
        }
        if (n.version < kMinVersion) {
            err = "libnccl.so.2 is version " + std::to_string(n.version) +
                  "; NCCL 2.14 or later is required (non-blocking communicators, abort, ncclAvg)";
            return;
        }
        if (!n.get_unique_id || !n.init_config || !n.comm_destroy || !n.comm_abort || !n.async_error ||
            !n.all_reduce)
            err = "libnccl.so.2 lacks an expected entry point";
    });
    if (!err.empty()) fail("nccl", err);
    return n;
}

std::string nccl_msg(ncclResult_t rc) {
    const Nccl& n = nccl();
    return std::string("NCCL error ") + std::to_string((int)rc) + ": " +
           (n.error_string ? n.error_string(rc) : "unknown");
}

// The library's communicator handle.
struct Comm {
    ncclComm_t comm = nullptr;
    int device = 0;
    int timeout_ms = 0;
    bool aborted = false;
};

Comm* as_comm(void* c, const char* where) {
    if (!c) fail(where, "null communicator");
    Comm* k = static_cast<Comm*>(c);
    if (k->aborted) fail(where, "the communicator was aborted after an earlier failure: make a new one");
    return k;
}

using clock_t_ = std::chrono::steady_clock;

// Abort (ends the communicator's kernels still waiting on the GPU) and raise.
[[noreturn]] void abort_and_fail(Comm* k, const char* where, const std::string& why) {
    if (!k->aborted) {
        nccl().comm_abort(k->comm);
        k->aborted = true;
    }
    fail(where, why);
}

// Poll a non-blocking communicator until its pending operation (set-up, or an
// enqueue that returned ncclInProgress) settles.
void settle(Comm* k, const char* where, clock_t_::time_point deadline) {
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t rc = nccl().async_error(k->comm, &st);
        if (rc != ncclSuccess) abort_and_fail(k, where, nccl_msg(rc));
        if (st == ncclSuccess) return;
        if (st != ncclInProgress) abort_and_fail(k, where, nccl_msg(st));
        if (clock_t_::now() > deadline)
            abort_and_fail(k, where, "timed out after " + std::to_string(k->timeout_ms) +
                                         " ms (a peer rank did not join); the communicator was aborted");
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

}  // namespace

void nccl_unique_id(void* out128) {
    ncclUniqueId id{};
    const ncclResult_t rc = nccl().get_unique_id(&id);
    if (rc != ncclSuccess) fail("bsml_nccl_unique_id", nccl_msg(rc));
    static_assert(sizeof(id.internal) == 128, "ncclUniqueId is 128 bytes");
    std::memcpy(out128, id.internal, 128);
}

void* nccl_comm_init(int nranks, const void* id128, int rank, int device, int timeout_ms) {
    if (nranks < 1 || rank < 0 || rank >= nranks) fail("bsml_nccl_comm_init", "bad rank or rank count");
    if (timeout_ms <= 0) fail("bsml_nccl_comm_init", "the timeout must be positive");
    BSML_CUDA(cudaSetDevice(device));
    ncclUniqueId id{};
    std::memcpy(id.internal, id128, 128);
    Comm* k = new Comm;
    k->device = device;
    k->timeout_ms = timeout_ms;
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const ncclResult_t rc = nccl().init_config(&k->comm, nranks, id, rank, &cfg);
    if (rc != ncclSuccess && rc != ncclInProgress) {
        if (k->comm) nccl().comm_abort(k->comm);
        delete k;
        fail("bsml_nccl_comm_init", nccl_msg(rc));
    }
    try {
        settle(k, "bsml_nccl_comm_init", clock_t_::now() + std::chrono::milliseconds(timeout_ms));
    } catch (...) {
        delete k;   // already aborted
        throw;
    }
    return k;
}

void nccl_comm_destroy(void* comm) {
    if (!comm) return;
    Comm* k = static_cast<Comm*>(comm);
    ncclResult_t rc = ncclSuccess;
    if (!k->aborted) {
        rc = nccl().comm_destroy(k->comm);
        if (rc == ncclInProgress) {   // non-blocking destroy: wait for it to finish (bounded)
            try {
                settle(k, "bsml_nccl_comm_destroy", clock_t_::now() + std::chrono::milliseconds(k->timeout_ms));
                rc = ncclSuccess;
            } catch (...) {
                delete k;
                throw;
            }
        }
    }
    delete k;
    if (rc != ncclSuccess) fail("bsml_nccl_comm_destroy", nccl_msg(rc));
}

void nccl_allreduce(void* comm, float* grads, int64_t n, bool average, cudaStream_t st) {
    Comm* k = as_comm(comm, "bsml_allreduce_grads");
    if (!grads || n < 0) fail("bsml_allreduce_grads", "bad argument");
    const ncclResult_t rc =
        nccl().all_reduce(grads, grads, (size_t)n, ncclFloat32, average ? ncclAvg : ncclSum, k->comm, st);
    if (rc == ncclInProgress)
        settle(k, "bsml_allreduce_grads", clock_t_::now() + std::chrono::milliseconds(k->timeout_ms));
    else if (rc != ncclSuccess)
        abort_and_fail(k, "bsml_allreduce_grads", nccl_msg(rc));
}

void nccl_sync(void* comm, cudaStream_t st) {
    Comm* k = as_comm(comm, "bsml_nccl_sync");
    const auto deadline = clock_t_::now() + std::chrono::milliseconds(k->timeout_ms);
    for (;;) {
        ncclResult_t as = ncclSuccess;
        const ncclResult_t rc = nccl().async_error(k->comm, &as);
        if (rc != ncclSuccess) abort_and_fail(k, "bsml_nccl_sync", nccl_msg(rc));
        if (as != ncclSuccess && as != ncclInProgress) abort_and_fail(k, "bsml_nccl_sync", nccl_msg(as));
        const cudaError_t q = cudaStreamQuery(st);
        if (q == cudaSuccess) return;
        if (q != cudaErrorNotReady) {
            (void)cudaGetLastError();
            abort_and_fail(k, "bsml_nccl_sync", std::string("CUDA error: ") + cudaGetErrorString(q));
        }
        if (clock_t_::now() > deadline)
            abort_and_fail(k, "bsml_nccl_sync", "the step's collectives did not finish within " +
                                                    std::to_string(k->timeout_ms) +
                                                    " ms (a peer rank left?); the communicator was aborted");
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

int nccl_version() { return nccl().version; }

}  // namespace bsml
