// Hankel windows with a pre-kernel rotary position encoding (reference
// FD/ROPE.py:31-106,231-345): the per-row preprocessing of the RoPE-DMAP
// encoder, after which fit and encode are the ordinary prepass / DMAP / AMAP
// passes on the rotated window vectors.
//
// Window T, sample c, feature j is read at F[T*sT + c*sC + j] and centred,
//   w = (F[..] - mu[j]) / sigma[j],
// its position at pos[T*pT + c*pC].  A time series gives the Hankel windows
// with sT = D, sC = step*D, pT = 1, pC = step (no copy of the windows is
// made); an explicit (B, L, D) window array has sT = L*D, sC = D.
//   sample mode: pairs (2p, 2p+1) of each sample rotate by
//                theta = pos(T, c) * pos_scale * freqs[p]         (p < D/2)
//   window mode: pairs (2p, 2p+1) of the flattened window (length Z = L*D)
//                rotate by theta = pos(T, c_w) * pos_scale * freqs[p]  (p < Z/2)
//   an odd last coordinate (of a sample, resp. of the window) is copied.
//
// One thread per output pair; fp64 arithmetic (positions times frequencies can
// reach 1e5 radians, where fp32 sin/cos keep no digits); fp32 output row-major
// (K, L*D).  HBM-bound elementwise kernel.
#include "fd_common.cuh"

namespace fd {
namespace rope {

__global__ void windows_kernel(const double* __restrict__ F, int64_t sT, int64_t sC, const double* __restrict__ pos,
                               int64_t pT, int64_t pC, int64_t K, int D, int L, int window_mode, int c_w,
                               double pos_scale, const double* __restrict__ freqs, int n_freqs,
                               const double* __restrict__ mu, const double* __restrict__ sigma,
                               float* __restrict__ Y) {
    const int Z = L * D;
    const int unit = window_mode ? (Z + 1) / 2 : L * ((D + 1) / 2);
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= K * unit) return;
    const int64_t T = g / unit;
    const int u = (int)(g - T * unit);
    int z0, p, cp;
    if (window_mode) {
        z0 = 2 * u;
        p = u;
        cp = c_w;
    } else {
        const int per = (D + 1) / 2;
        cp = u / per;
        p = u - cp * per;
        z0 = cp * D + 2 * p;
    }
    auto wval = [&](int z) {
        const int c = z / D, j = z - c * D;
        return (F[T * sT + c * sC + j] - mu[j]) / sigma[j];
    };
    const bool pair = window_mode ? (z0 + 1 < Z) : (2 * p + 1 < D);
    float* y = Y + T * (int64_t)Z + z0;
    if (!pair) {
        y[0] = (float)wval(z0);
        return;
    }
    const double a = wval(z0), b = wval(z0 + 1);
    const double f = p < n_freqs ? freqs[p] : 0.0;
    double s, c;
    sincos(pos[T * pT + cp * pC] * pos_scale * f, &s, &c);
    y[0] = (float)(a * c - b * s);
    y[1] = (float)(a * s + b * c);
}

}  // namespace rope
}  // namespace fd

extern "C" int fd_rope_windows(const double* F, int64_t sT, int64_t sC, const double* pos, int64_t pT, int64_t pC,
                               int64_t K, int D, int L, int window_mode, int c_w, double pos_scale,
                               const double* freqs, int n_freqs, const double* mu, const double* sigma, float* Y,
                               void* stream) {
    FD_CHECK_ARG(K >= 0 && D >= 1 && L >= 1, "fd_rope_windows: K=%lld D=%d L=%d", (long long)K, D, L);
    FD_CHECK_ARG(c_w >= 0 && c_w < L, "fd_rope_windows: c_w=%d not in [0, L)", c_w);
    FD_CHECK_ARG(n_freqs >= 0, "fd_rope_windows: n_freqs=%d", n_freqs);
    if (K == 0) return FD_OK;
    FD_CHECK_ARG(F && pos && mu && sigma && Y && (n_freqs == 0 || freqs), "fd_rope_windows: null pointer");
    const int Z = L * D;
    const int unit = window_mode ? (Z + 1) / 2 : L * ((D + 1) / 2);
    const int64_t total = K * unit;
    fd::rope::windows_kernel<<<(unsigned)fd::cdiv(total, 256), 256, 0, (cudaStream_t)stream>>>(
        F, sT, sC, pos, pT, pC, K, D, L, window_mode ? 1 : 0, c_w, pos_scale, freqs, n_freqs, mu, sigma, Y);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}
