// Lanczos vector operations on the device: the full fp64 reorthogonalisation
// of one Lanczos step against the Krylov basis, with its norm, in three
// passes over the basis and no host synchronisation.
//
// The reference keeps the Krylov basis and its reorthogonalisation in fp64 on
// the host inside ARPACK (FD/eigensolver.py:17-20, 69-76).  Here the basis V
// is a row-major [rows][ldv] fp64 array in device memory (row i = Lanczos
// vector i, each of n entries), and one step turns the operator output w into
// the next basis vector:
//
//   pass A   h1 = V w                                  (dots)
//   pass B   w1 = w - V^T h1,   h2 = V w1,   s = ||w1||^2
//   pass C   beta = sqrt(s - ||h2||^2),  out = (w1 - V^T h2) / beta
//
// which is classical Gram-Schmidt applied twice (CGS2) with the norm of the
// twice-orthogonalised vector taken from Pythagoras (V has orthonormal rows,
// so ||w1 - V^T h2||^2 = ||w1||^2 - ||h2||^2 to rounding).  The coefficients
// h1 + h2 and beta go to a device array the caller reads once per restart.
//
// Every reduction runs in a fixed order (per-block partials, then one block
// per coefficient summing the partials in block order), so results are
// bit-reproducible.  Pass B keeps its chunk of V in shared memory, so each
// pass reads the basis from memory once: 3 rows n + O(n) fp64 words per step.
#include "fd_common.cuh"

namespace fd {
namespace lz {

constexpr int CHUNK = 256;     // entries of n per block (one per thread)
constexpr int THREADS = CHUNK;
constexpr int WARPS = THREADS / 32;
// pass B keeps its chunk of every basis row in shared memory: 128 entries per
// block (96 rows x 128 x 8 B = 96 KB at most) so that two or three blocks share
// an SM; passes A and C, which need no such copy, take 256
constexpr int CHUNK_B = 128;
constexpr int WARPS_B = CHUNK_B / 32;
constexpr int MAX_ROWS = 96;   // basis rows a step orthogonalises against

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ int chunk_count(int64_t n, int64_t base) {
    return (int)(n - base < CHUNK ? n - base : CHUNK);
}

// pass A: part[i][blk] = V[i][chunk] . w[chunk]
__global__ void __launch_bounds__(THREADS) pass_a_kernel(const double* __restrict__ V, int64_t ldv, int rows,
                                                         int64_t n, const double* __restrict__ w,
                                                         double* __restrict__ part) {
    __shared__ double sw[CHUNK];
    const int64_t base = (int64_t)blockIdx.x * CHUNK;
    const int cnt = chunk_count(n, base);
    const int t = threadIdx.x;
    if (t < cnt) sw[t] = w[base + t];
    __syncthreads();
    const int warp = t >> 5, lane = t & 31;
    for (int i = warp; i < rows; i += WARPS) {
        const double* vr = V + (int64_t)i * ldv + base;
        double acc = 0.0;
        for (int e = lane; e < cnt; e += 32) acc += vr[e] * sw[e];
        acc = warp_sum(acc);
        if (lane == 0) part[(int64_t)i * gridDim.x + blockIdx.x] = acc;
    }
}

// out[i] = sum over blocks of part[i][blk], in block order; one block per row.
__global__ void __launch_bounds__(THREADS) reduce_kernel(const double* __restrict__ part, int nparts,
                                                         double* __restrict__ out) {
    __shared__ double red[THREADS];
    const int i = blockIdx.x;
    double acc = 0.0;
    for (int b = threadIdx.x; b < nparts; b += THREADS) acc += part[(int64_t)i * nparts + b];
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int s = THREADS / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) out[i] = red[0];
}

// pass B: w1 = w - V^T h1 (written to w); part = V w1, and ||w1||^2 in row `rows`
__global__ void __launch_bounds__(CHUNK_B) pass_b_kernel(const double* __restrict__ V, int64_t ldv, int rows,
                                                         int64_t n, double* __restrict__ w,
                                                         const double* __restrict__ h1, double* __restrict__ part) {
    extern __shared__ double smem[];
    double* sV = smem;                         // [rows][CHUNK_B]
    double* sw = sV + (size_t)rows * CHUNK_B;  // [CHUNK_B]
    double* sh = sw + CHUNK_B;                 // [rows]
    const int64_t base = (int64_t)blockIdx.x * CHUNK_B;
    const int cnt = (int)(n - base < CHUNK_B ? n - base : CHUNK_B);
    const int t = threadIdx.x;
    for (int i = t; i < rows; i += CHUNK_B) sh[i] = h1[i];
    for (int i = 0; i < rows; ++i) sV[i * CHUNK_B + t] = t < cnt ? V[(int64_t)i * ldv + base + t] : 0.0;
    __syncthreads();
    double x = t < cnt ? w[base + t] : 0.0;
    for (int i = 0; i < rows; ++i) x -= sV[i * CHUNK_B + t] * sh[i];
    sw[t] = x;
    if (t < cnt) w[base + t] = x;
    __syncthreads();
    const int warp = t >> 5, lane = t & 31;
    for (int i = warp; i <= rows; i += WARPS_B) {
        double acc = 0.0;
        for (int e = lane; e < cnt; e += 32) {
            const double xe = sw[e];
            acc += (i < rows ? sV[i * CHUNK_B + e] : xe) * xe;
        }
        acc = warp_sum(acc);
        if (lane == 0) part[(int64_t)i * gridDim.x + blockIdx.x] = acc;
    }
}

// pass C: beta = sqrt(s - ||h2||^2); out = (w1 - V^T h2) / beta (zeros if
// beta <= 1e-300); coef[i] += h2[i], coef[rows] = beta.
__global__ void __launch_bounds__(THREADS) pass_c_kernel(const double* __restrict__ V, int64_t ldv, int rows,
                                                         int64_t n, const double* __restrict__ w,
                                                         const double* __restrict__ h2s, double* __restrict__ out,
                                                         double* __restrict__ coef) {
    __shared__ double sh[MAX_ROWS];
    __shared__ double sbeta;
    const int t = threadIdx.x;
    for (int i = t; i < rows; i += THREADS) sh[i] = h2s[i];
    if (t == 0) {
        double q = 0.0;
        for (int i = 0; i < rows; ++i) q += h2s[i] * h2s[i];
        const double b2 = h2s[rows] - q;
        sbeta = b2 > 0.0 ? sqrt(b2) : 0.0;
    }
    __syncthreads();
    const double beta = sbeta;
    const double inv = beta > 1e-300 ? 1.0 / beta : 0.0;
    const int64_t e = (int64_t)blockIdx.x * CHUNK + t;
    if (e < n) {
        double x = w[e];
        for (int i = 0; i < rows; ++i) x -= V[(int64_t)i * ldv + e] * sh[i];
        out[e] = x * inv;
    }
    if (blockIdx.x == 0) {
        for (int i = t; i < rows; i += THREADS) coef[i] += sh[i];
        if (t == 0) coef[rows] = beta;
    }
}

}  // namespace lz
}  // namespace fd

using namespace fd;

extern "C" size_t fd_lanczos_workspace_bytes(int64_t n, int rows) {
    if (n < 1 || rows < 0) return 0;
    const int64_t nblk = cdiv(n, lz::CHUNK_B);   // the larger partial count (pass B)
    return align256(sizeof(double) * (size_t)nblk * (rows + 1)) + align256(sizeof(double) * (rows + 1));
}

extern "C" int fd_lanczos_reorth(const double* V, int64_t ldv, int rows, int64_t n, double* w, double* out,
                                 double* coef, void* workspace, size_t workspace_bytes, void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    FD_CHECK_ARG(n >= 1 && rows >= 1 && rows <= lz::MAX_ROWS, "fd_lanczos_reorth: n=%lld rows=%d (rows 1..%d)",
                 (long long)n, rows, lz::MAX_ROWS);
    FD_CHECK_ARG(ldv >= n, "fd_lanczos_reorth: ldv=%lld < n=%lld", (long long)ldv, (long long)n);
    FD_CHECK_ARG(V && w && out && coef, "fd_lanczos_reorth: null pointer");
    const size_t need = fd_lanczos_workspace_bytes(n, rows);
    if (workspace_bytes < need)
        return set_error(FD_ERR_WORKSPACE, "fd_lanczos_reorth: workspace %zu B < required %zu B", workspace_bytes,
                         need);
    FD_CHECK_ARG(workspace && ((uintptr_t)workspace & 255) == 0, "workspace must be non-null and 256-byte aligned");
    const int nblk = (int)cdiv(n, lz::CHUNK);
    const int nblk_b = (int)cdiv(n, lz::CHUNK_B);
    double* part = (double*)workspace;
    double* h2s = (double*)((uint8_t*)workspace + align256(sizeof(double) * (size_t)nblk_b * (rows + 1)));
    const size_t smem_b = sizeof(double) * ((size_t)rows * lz::CHUNK_B + lz::CHUNK_B + rows);
    FD_CUDA_TRY(cudaFuncSetAttribute(lz::pass_b_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_b));
    lz::pass_a_kernel<<<nblk, lz::THREADS, 0, s>>>(V, ldv, rows, n, w, part);
    lz::reduce_kernel<<<rows, lz::THREADS, 0, s>>>(part, nblk, coef);
    lz::pass_b_kernel<<<nblk_b, lz::CHUNK_B, smem_b, s>>>(V, ldv, rows, n, w, coef, part);
    lz::reduce_kernel<<<rows + 1, lz::THREADS, 0, s>>>(part, nblk_b, h2s);
    lz::pass_c_kernel<<<nblk, lz::THREADS, 0, s>>>(V, ldv, rows, n, w, h2s, out, coef);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}
