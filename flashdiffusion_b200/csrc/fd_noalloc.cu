// fd_apply_noalloc: the 16-bit tensor-core operator with its scratch memory in
// a fixed, library-owned device array instead of a caller workspace.
//
// Who needs this: callers that cannot call cudaMalloc, or cannot hand this
// library a device buffer of their own — for example a host that binds the
// library through a foreign-function interface with no device allocator to
// pass in, or a process whose device memory is entirely owned by a pre-sized
// pool that forbids allocations outside it, or a latency-critical loop that
// must not pay the implicit device synchronisation of cudaMalloc/cudaFree.
// Such a caller still provides the packed operands, the right-hand side and
// the output; only the scratch (the prepared right-hand side and the
// cross-CTA partial sums) comes from here.
//
// The scratch is one file-scope __device__ array of FD_NOALLOC_SCRATCH_BYTES.
// Every GPU that loads the library holds it until the process exits.  Its
// device address is looked up once per device with cudaGetSymbolAddress (the
// array's name in host code is only a host-side stand-in, not a device
// address), on the first call made with that device current.
#include <mutex>

#include "fd_prep.cuh"

namespace fd {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[FD_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device (looked up once).
int noalloc_scratch(void** ptr) {
    int dev = 0;
    FD_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return set_error(FD_ERR_ARG, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return set_error(FD_ERR_CUDA, "fd_apply_noalloc: cudaGetSymbolAddress of the static scratch failed: %s",
                             cudaGetErrorString(e));
        g_noalloc_addr[dev] = p;
    }
    *ptr = g_noalloc_addr[dev];
    return FD_OK;
}

}  // namespace
}  // namespace fd

extern "C" int fd_apply_noalloc(const void* Qop, int64_t nq, const void* Kop, int64_t nk, int d, int tile,
                                const void* V, int v_dtype, int r, const float* col_scale, const float* col_h,
                                const float* row_scale, const float* row_div, void* out, int out_dtype,
                                void* stream) {
    using namespace fd;
    FD_CHECK_ARG(tile == FD_TILE_F16 || tile == FD_TILE_BF16,
                 "fd_apply_noalloc: only the 16-bit tensor-core tiles (FD_TILE_F16 / FD_TILE_BF16) are supported");
    FD_CHECK_ARG(nq >= 0 && nk >= 0 && r >= 1, "fd_apply_noalloc: bad shape nq=%lld nk=%lld r=%d",
                 (long long)nq, (long long)nk, r);
    const size_t need = fd_apply_workspace_bytes(nq, nk, r, tile);
    if (need > (size_t)FD_NOALLOC_SCRATCH_BYTES) {
        // the kernel's cross-CTA partial sums grow with r but not with nk; the
        // rest of the scratch is the prepared right-hand side, linear in nk
        const size_t fixed = fd_apply_workspace_bytes(nq, 0, r, tile);
        return set_error(FD_ERR_WORKSPACE,
                         "fd_apply_noalloc: nk=%lld, r=%d needs %zu B of scratch (%zu B of it even for one key) but "
                         "the static scratch holds %zu B; limits on a 148-SM GPU: r=1 up to about 1.9 million keys, "
                         "r=2..16 up to about 55,000 keys, r>=17 not supported; use fd_apply with a workspace",
                         (long long)nk, r, need, fixed, (size_t)FD_NOALLOC_SCRATCH_BYTES);
    }
    void* scratch = nullptr;
    FD_TRY(noalloc_scratch(&scratch));
    // Nothing in the scratch has to start at zero: the right-hand side region
    // (including its zero padding) and every partial-sum slot the fix-up pass
    // reads are written earlier in the same call, and the tile launch clears
    // its lockstep pacing counter itself.
    return fd_apply(Qop, nq, Kop, nk, d, tile, V, v_dtype, r, col_scale, col_h, row_scale, row_div, out,
                    out_dtype, scratch, (size_t)FD_NOALLOC_SCRATCH_BYTES, stream);
}
