// fd_comm_*: the one collective of the row-sharded operator, for hosts that
// call the C ABI directly (no torch.distributed).  Each rank owns contiguous
// row shards of Q and holds all of K; after its tile pass it all-gathers the
// output shards so every rank holds the full product (the Lanczos / LOBPCG
// update is then replicated on every rank, no further collective).
//
// NCCL is opened at run time (dlopen of libnccl.so.2, which resolves to the
// copy a host process has already loaded, e.g. torch's), so the operator
// library itself loads and runs without NCCL; only these entry points need it.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "fd_common.cuh"

namespace fd {
namespace {

struct Nccl {
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*abort)(ncclComm_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

std::mutex g_nccl_mu;
Nccl g_nccl;

int nccl(const Nccl** out) {
    std::lock_guard<std::mutex> lock(g_nccl_mu);
    if (!g_nccl.ok) {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return set_error(FD_ERR_UNSUPPORTED, "fd_comm: NCCL not found (dlopen libnccl.so.2: %s)", dlerror());
        Nccl n;
        n.get_unique_id = (decltype(n.get_unique_id))dlsym(h, "ncclGetUniqueId");
        n.init_rank = (decltype(n.init_rank))dlsym(h, "ncclCommInitRank");
        n.all_gather = (decltype(n.all_gather))dlsym(h, "ncclAllGather");
        n.abort = (decltype(n.abort))dlsym(h, "ncclCommAbort");
        n.destroy = (decltype(n.destroy))dlsym(h, "ncclCommDestroy");
        n.async_error = (decltype(n.async_error))dlsym(h, "ncclCommGetAsyncError");
        n.error_string = (decltype(n.error_string))dlsym(h, "ncclGetErrorString");
        if (!n.get_unique_id || !n.init_rank || !n.all_gather || !n.abort || !n.destroy || !n.async_error ||
            !n.error_string)
            return set_error(FD_ERR_UNSUPPORTED, "fd_comm: the NCCL library lacks an expected symbol");
        n.ok = true;
        g_nccl = n;
    }
    *out = &g_nccl;
    return FD_OK;
}

#define FD_NCCL_TRY(n, expr)                                                                    \
    do {                                                                                        \
        ncclResult_t _r = (expr);                                                               \
        if (_r != ncclSuccess)                                                                  \
            return ::fd::set_error(FD_ERR_CUDA, "fd_comm: %s failed: %s", #expr, (n)->error_string(_r)); \
    } while (0)

}  // namespace
}  // namespace fd

using namespace fd;

extern "C" size_t fd_comm_id_bytes(void) { return sizeof(ncclUniqueId); }

extern "C" int fd_comm_get_id(void* id) {
    FD_CHECK_ARG(id, "fd_comm_get_id: null id");
    const Nccl* n = nullptr;
    FD_TRY(nccl(&n));
    ncclUniqueId u;
    FD_NCCL_TRY(n, n->get_unique_id(&u));
    memcpy(id, &u, sizeof(u));
    return FD_OK;
}

extern "C" int fd_comm_init(void** comm, const void* id, int nranks, int rank) {
    FD_CHECK_ARG(comm && id, "fd_comm_init: null pointer");
    FD_CHECK_ARG(nranks >= 1 && rank >= 0 && rank < nranks, "fd_comm_init: rank %d of %d", rank, nranks);
    const Nccl* n = nullptr;
    FD_TRY(nccl(&n));
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    ncclComm_t c = nullptr;
    FD_NCCL_TRY(n, n->init_rank(&c, nranks, u, rank));
    *comm = (void*)c;
    return FD_OK;
}

extern "C" int fd_comm_allgather(void* comm, const void* send, void* recv, size_t bytes_per_rank, void* stream) {
    FD_CHECK_ARG(comm, "fd_comm_allgather: null comm");
    FD_CHECK_ARG(bytes_per_rank == 0 || (send && recv), "fd_comm_allgather: null buffer");
    const Nccl* n = nullptr;
    FD_TRY(nccl(&n));
    FD_NCCL_TRY(n, n->all_gather(send, recv, bytes_per_rank, ncclInt8, (ncclComm_t)comm, (cudaStream_t)stream));
    return FD_OK;
}

extern "C" int fd_comm_check(void* comm) {
    FD_CHECK_ARG(comm, "fd_comm_check: null comm");
    const Nccl* n = nullptr;
    FD_TRY(nccl(&n));
    ncclResult_t st = ncclSuccess;
    FD_NCCL_TRY(n, n->async_error((ncclComm_t)comm, &st));
    if (st != ncclSuccess && st != ncclInProgress)
        return set_error(FD_ERR_CUDA, "fd_comm: asynchronous NCCL error: %s", n->error_string(st));
    return FD_OK;
}

extern "C" int fd_comm_abort(void* comm) {
    if (!comm) return FD_OK;
    const Nccl* n = nullptr;
    FD_TRY(nccl(&n));
    FD_NCCL_TRY(n, n->abort((ncclComm_t)comm));
    return FD_OK;
}

extern "C" int fd_comm_destroy(void* comm) {
    if (!comm) return FD_OK;
    const Nccl* n = nullptr;
    FD_TRY(nccl(&n));
    FD_NCCL_TRY(n, n->destroy((ncclComm_t)comm));
    return FD_OK;
}
