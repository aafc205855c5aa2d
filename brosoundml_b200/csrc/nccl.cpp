// Data-parallel gradient averaging for C / C++ callers without torch: NCCL is
// loaded at run time (libnccl.so.2 — the copy already in the process when there is
// one), so the library has no link-time NCCL dependency. One process per GPU; the
// flat gradient buffer is all-reduced once per step (sum, or average over ranks).
#include <dlfcn.h>

#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "nccl_dl.h"

namespace bsml {

namespace {

// the few NCCL entry points used, with their C signatures (nccl.h)
struct UniqueId {
    char internal[128];
};
using ncclComm_t = void*;
using fn_get_unique_id = int (*)(UniqueId*);
using fn_comm_init_rank = int (*)(ncclComm_t*, int, UniqueId, int);
using fn_comm_destroy = int (*)(ncclComm_t);
using fn_all_reduce = int (*)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t);
using fn_error_string = const char* (*)(int);

constexpr int kNcclFloat32 = 7;   // ncclDataType_t::ncclFloat32
constexpr int kNcclSum = 0;       // ncclRedOp_t::ncclSum
constexpr int kNcclAvg = 4;       // ncclRedOp_t::ncclAvg (NCCL >= 2.10)

struct Nccl {
    void* h = nullptr;
    fn_get_unique_id get_unique_id = nullptr;
    fn_comm_init_rank comm_init_rank = nullptr;
    fn_comm_destroy comm_destroy = nullptr;
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
        n.get_unique_id = reinterpret_cast<fn_get_unique_id>(dlsym(h, "ncclGetUniqueId"));
        n.comm_init_rank = reinterpret_cast<fn_comm_init_rank>(dlsym(h, "ncclCommInitRank"));
        n.comm_destroy = reinterpret_cast<fn_comm_destroy>(dlsym(h, "ncclCommDestroy"));
        n.all_reduce = reinterpret_cast<fn_all_reduce>(dlsym(h, "ncclAllReduce"));
        n.error_string = reinterpret_cast<fn_error_string>(dlsym(h, "ncclGetErrorString"));
        if (!n.get_unique_id || !n.comm_init_rank || !n.comm_destroy || !n.all_reduce)
            err = "libnccl.so.2 lacks an expected entry point";
    });
    if (!err.empty()) fail("nccl", err);
    return n;
}

void check_nccl(int rc, const char* where) {
    if (rc != 0) {
        const Nccl& n = nccl();
        fail(where, std::string("NCCL error ") + std::to_string(rc) + ": " +
                        (n.error_string ? n.error_string(rc) : "unknown"));
    }
}

}  // namespace

void nccl_unique_id(void* out128) {
    UniqueId id{};
    check_nccl(nccl().get_unique_id(&id), "bsml_nccl_unique_id");
    std::memcpy(out128, id.internal, 128);
}

void* nccl_comm_init(int nranks, const void* id128, int rank, int device) {
    if (nranks < 1 || rank < 0 || rank >= nranks) fail("bsml_nccl_comm_init", "bad rank or rank count");
    BSML_CUDA(cudaSetDevice(device));
    UniqueId id{};
    std::memcpy(id.internal, id128, 128);
    ncclComm_t comm = nullptr;
    check_nccl(nccl().comm_init_rank(&comm, nranks, id, rank), "bsml_nccl_comm_init");
    return comm;
}

void nccl_comm_destroy(void* comm) {
    if (comm) check_nccl(nccl().comm_destroy(comm), "bsml_nccl_comm_destroy");
}

void nccl_allreduce(void* comm, float* grads, int64_t n, bool average, cudaStream_t st) {
    if (!comm || !grads || n < 0) fail("bsml_allreduce_grads", "bad argument");
    check_nccl(nccl().all_reduce(grads, grads, (size_t)n, kNcclFloat32, average ? kNcclAvg : kNcclSum, comm, st),
               "bsml_allreduce_grads");
}

}  // namespace bsml
