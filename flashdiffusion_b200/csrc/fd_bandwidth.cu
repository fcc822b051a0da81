// Bandwidth selection on the GPU (reference: FD/utils.py:16-52).
//
//   fd_knn_sqdist      the k smallest squared distances of every query row to a
//                      key set (self-tuning bandwidth sigma_i = sqrt of the k-th,
//                      FD/utils.py:31-52, whose host version sorts a dense N x N
//                      distance matrix)
//   fd_pairwise_sqdist all squared distances of a small sample (the median
//                      heuristic, FD/utils.py:16-28, takes the median of the
//                      positive ones)
//
// Both are fp32 CUDA-core kernels on coordinate differences (not the law of
// cosines): the nearest-neighbour distances are the small ones, where the
// cancellation of |x|^2 + |y|^2 - 2 x.y would cost the most digits, and the
// 16-bit tensor-core operands would leave a relative error of ~|x|^2 2^-11 / d^2.
//
// knn_kernel: one thread per query row (128 rows per CTA); key tiles of KT rows
// staged in shared memory ([KT][dp], dp = d rounded up to 4, zero padded) and
// read as broadcast float4; KT accumulators per thread; the KMAX smallest
// values so far kept sorted in registers and updated by a branch-free
// min/max insertion only when a candidate beats the current KMAX-th.
#include <cfloat>

#include "fd_common.cuh"

namespace fd {
namespace bw {

constexpr int ROWS = 128;
constexpr int KT = 32;

template <int KMAX>
__global__ void __launch_bounds__(ROWS) knn_kernel(const float* __restrict__ Q, int64_t nq,
                                                   const float* __restrict__ K, int64_t nk, int d, int dp, int k,
                                                   float* __restrict__ out) {
    extern __shared__ float4 ks4[];
    float* ks = reinterpret_cast<float*>(ks4);
    const int64_t i = (int64_t)blockIdx.x * ROWS + threadIdx.x;
    const bool valid = i < nq;
    const float* q = Q + (valid ? i : 0) * (int64_t)d;
    float best[KMAX];
#pragma unroll
    for (int s = 0; s < KMAX; ++s) best[s] = FLT_MAX;
    for (int64_t j0 = 0; j0 < nk; j0 += KT) {
        const int nt = (nk - j0 < KT) ? (int)(nk - j0) : KT;
        __syncthreads();
        for (int e = threadIdx.x; e < KT * dp; e += ROWS) {
            const int j = e / dp, c = e - j * dp;
            ks[e] = (j < nt && c < d) ? K[(j0 + j) * (int64_t)d + c] : 0.f;
        }
        __syncthreads();
        float acc[KT];
#pragma unroll
        for (int j = 0; j < KT; ++j) acc[j] = 0.f;
        for (int c = 0; c < dp; c += 4) {
            const float q0 = c < d ? q[c] : 0.f, q1 = c + 1 < d ? q[c + 1] : 0.f;
            const float q2 = c + 2 < d ? q[c + 2] : 0.f, q3 = c + 3 < d ? q[c + 3] : 0.f;
#pragma unroll
            for (int j = 0; j < KT; ++j) {
                const float4 kv = ks4[(j * dp + c) >> 2];
                const float t0 = q0 - kv.x, t1 = q1 - kv.y, t2 = q2 - kv.z, t3 = q3 - kv.w;
                acc[j] = fmaf(t0, t0, acc[j]);
                acc[j] = fmaf(t1, t1, acc[j]);
                acc[j] = fmaf(t2, t2, acc[j]);
                acc[j] = fmaf(t3, t3, acc[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < KT; ++j) {
            float x = acc[j];
            if (j < nt && x < best[KMAX - 1]) {
#pragma unroll
                for (int s = 0; s < KMAX; ++s) {
                    const float lo = fminf(best[s], x);
                    x = fmaxf(best[s], x);
                    best[s] = lo;
                }
            }
        }
    }
    if (valid) {
#pragma unroll
        for (int s = 0; s < KMAX; ++s)
            if (s < k) out[i * k + s] = best[s];
    }
}

__global__ void pairwise_kernel(const float* __restrict__ X, int64_t m, int d, float* __restrict__ out) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t i = blockIdx.y;
    if (j >= m) return;
    const float* a = X + i * d;
    const float* b = X + j * d;
    float acc = 0.f;
    for (int c = 0; c < d; ++c) {
        const float t = a[c] - b[c];
        acc = fmaf(t, t, acc);
    }
    out[i * m + j] = acc;
}

template <int KMAX>
static int launch_knn(const float* Q, int64_t nq, const float* K, int64_t nk, int d, int k, float* out,
                      cudaStream_t s) {
    const int dp = (int)round_up(d, 4);
    const size_t smem = sizeof(float) * KT * dp;
    FD_CUDA_TRY(cudaFuncSetAttribute(knn_kernel<KMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    knn_kernel<KMAX><<<(unsigned)cdiv(nq, ROWS), ROWS, smem, s>>>(Q, nq, K, nk, d, dp, k, out);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

}  // namespace bw
}  // namespace fd

extern "C" {

int fd_knn_sqdist(const float* Q, int64_t nq, const float* K, int64_t nk, int d, int k, float* out,
                  void* stream) {
    FD_CHECK_ARG(nq >= 0 && nk >= 0, "fd_knn_sqdist: negative size");
    FD_CHECK_ARG(d >= 1 && d <= 1024, "fd_knn_sqdist: d = %d (1..1024)", d);
    FD_CHECK_ARG(k >= 1 && k <= 64, "fd_knn_sqdist: k = %d (1..64)", k);
    FD_CHECK_ARG(k <= nk, "fd_knn_sqdist: k = %d > %lld keys", k, (long long)nk);
    if (nq == 0) return FD_OK;
    FD_CHECK_ARG(Q && K && out, "fd_knn_sqdist: null pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (k <= 8) return fd::bw::launch_knn<8>(Q, nq, K, nk, d, k, out, s);
    if (k <= 16) return fd::bw::launch_knn<16>(Q, nq, K, nk, d, k, out, s);
    if (k <= 32) return fd::bw::launch_knn<32>(Q, nq, K, nk, d, k, out, s);
    return fd::bw::launch_knn<64>(Q, nq, K, nk, d, k, out, s);
}

int fd_pairwise_sqdist(const float* X, int64_t m, int d, float* out, void* stream) {
    FD_CHECK_ARG(m >= 0 && m <= 65535, "fd_pairwise_sqdist: m = %lld (0..65535)", (long long)m);
    FD_CHECK_ARG(d >= 1, "fd_pairwise_sqdist: d = %d", d);
    if (m == 0) return FD_OK;
    FD_CHECK_ARG(X && out, "fd_pairwise_sqdist: null pointer");
    dim3 grid((unsigned)fd::cdiv(m, 128), (unsigned)m);
    fd::bw::pairwise_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>(X, m, d, out);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

}  // extern "C"
