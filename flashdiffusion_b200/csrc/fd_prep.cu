// O(N) kernels around the O(N^2) tile kernels: norms, centring, operand
// packing, right-hand-side preparation and Coifman-Lafon normalisation.
// All of them are memory-bound one-pass kernels.
#include "fd_prep.cuh"

namespace fd {

__global__ void sq_norms_kernel(const void* __restrict__ X, int dtype, int64_t n, int d,
                                float* __restrict__ sq) {
    // one warp per row, lanes stride the columns
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    float s = 0.f;
    for (int k = lane; k < d; k += 32) {
        const float v = (float)load_as_f64(X, dtype, row * d + k);
        s = fmaf(v, v, s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) sq[row] = s;
}

// Column means of a strided subsample of at most `cap` rows (any shift is
// exact for a translation-invariant kernel; the mean only minimises rounding).
__global__ void mean_rows_kernel(const void* __restrict__ X, int dtype, int64_t n, int d,
                                 int64_t stride, int64_t cnt, float* __restrict__ shift) {
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        double s = 0.0;
        for (int64_t i = 0; i < cnt; ++i) s += load_as_f64(X, dtype, (i * stride) * d + c);
        shift[c] = (float)(s / (double)cnt);
    }
}

// 16-bit element conversion helpers (round to nearest)
struct H16 {
    typedef __half T;
    static __device__ __forceinline__ T from(double x) { return __float2half_rn((float)x); }
    static __device__ __forceinline__ double to(T v) { return (double)__half2float(v); }
    static constexpr double kMax = 65504.0;
};
struct B16 {
    typedef __nv_bfloat16 T;
    static __device__ __forceinline__ T from(double x) { return __double2bfloat16(x); }
    static __device__ __forceinline__ double to(T v) { return (double)__bfloat162float(v); }
    static constexpr double kMax = 3.0e38;
};

// Packed 16-bit operand (layout documented in fd_common.cuh).  One warp per
// row.  When a value of the row exceeds the 16-bit range, FD_ERR_RANGE is
// recorded in *status (the caller then repacks with the wider bf16 format).
template <class F>
__global__ void pack16_kernel(const void* __restrict__ X, int dtype, int64_t n, int d,
                              const float* __restrict__ shift, double s, int side, int kd,
                              typename F::T* __restrict__ out, int* __restrict__ status) {
    typedef typename F::T T;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    T* o = out + row * kd;
    double ss = 0.0, amax = 0.0;
    for (int k = lane; k < d; k += 32) {
        double x = load_as_f64(X, dtype, row * d + k);
        if (shift) x -= (double)shift[k];
        const T b = F::from(x * s);
        const double bv = F::to(b);
        ss += bv * bv;
        amax = fmax(amax, fabs(x * s));
        o[k] = b;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        ss += __shfl_xor_sync(0xffffffffu, ss, off);
        amax = fmax(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    }
    if (lane == 0) {
        const double nrm = -0.5 * ss;
        const T hi = F::from(nrm);
        const double r1 = nrm - F::to(hi);
        const T mid = F::from(r1);
        const T lo = F::from(r1 - F::to(mid));
        if (amax > 0.99 * F::kMax || -nrm > 0.99 * F::kMax || !(ss == ss)) atomicExch(status, FD_ERR_RANGE);
        const T one = F::from(1.0);
        if (side == FD_SIDE_QUERY) {
            o[d + 0] = one; o[d + 1] = one; o[d + 2] = one;
            o[d + 3] = hi; o[d + 4] = mid; o[d + 5] = lo;
        } else {
            o[d + 0] = hi; o[d + 1] = mid; o[d + 2] = lo;
            o[d + 3] = one; o[d + 4] = one; o[d + 5] = one;
        }
    }
    for (int k = d + 6 + lane; k < kd; k += 32) o[k] = F::from(0.0);
}

// fp32-class operand: every coordinate split into fp16 hi + lo (layout in
// fd_common.cuh, kd_f16x3); the norm is that of the split point hi + lo.
__global__ void pack_f16x3_kernel(const void* __restrict__ X, int dtype, int64_t n, int d,
                                  const float* __restrict__ shift, double s, int side, int kd,
                                  __half* __restrict__ out, int* __restrict__ status) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    __half* o = out + row * kd;
    double ss = 0.0, amax = 0.0;
    for (int k = lane; k < d; k += 32) {
        double x = load_as_f64(X, dtype, row * d + k);
        if (shift) x -= (double)shift[k];
        x *= s;
        const __half hi = H16::from(x);
        const __half lo = H16::from(x - H16::to(hi));
        const double a = H16::to(hi) + H16::to(lo);
        ss += a * a;
        amax = fmax(amax, fabs(x));
        o[k] = hi;
        if (side == FD_SIDE_QUERY) { o[d + k] = hi; o[2 * d + k] = lo; }
        else { o[d + k] = lo; o[2 * d + k] = hi; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        ss += __shfl_xor_sync(0xffffffffu, ss, off);
        amax = fmax(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    }
    const int e = 3 * d;
    if (lane == 0) {
        const double nrm = -0.5 * ss;
        const __half hi = H16::from(nrm);
        const double r1 = nrm - H16::to(hi);
        const __half mid = H16::from(r1);
        const __half lo = H16::from(r1 - H16::to(mid));
        if (amax > 0.99 * H16::kMax || -nrm > 0.99 * H16::kMax || !(ss == ss)) atomicExch(status, FD_ERR_RANGE);
        const __half one = H16::from(1.0);
        if (side == FD_SIDE_QUERY) {
            o[e + 0] = one; o[e + 1] = one; o[e + 2] = one;
            o[e + 3] = hi; o[e + 4] = mid; o[e + 5] = lo;
        } else {
            o[e + 0] = hi; o[e + 1] = mid; o[e + 2] = lo;
            o[e + 3] = one; o[e + 4] = one; o[e + 5] = one;
        }
    }
    for (int k = e + 6 + lane; k < kd; k += 32) o[k] = H16::from(0.0);
}

// fp32 operand: centred points scaled by sqrt(beta) [n][dp], then n squared
// norms of the stored values.  One warp per row.
__global__ void pack_f32_kernel(const void* __restrict__ X, int dtype, int64_t n, int d,
                                const float* __restrict__ shift, double sb, int dp,
                                float* __restrict__ pts, float* __restrict__ sq) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    float s = 0.f;
    for (int k = lane; k < dp; k += 32) {
        float x = 0.f;
        if (k < d) {
            double xv = load_as_f64(X, dtype, row * d + k);
            if (shift) xv -= (double)shift[k];
            x = (float)(xv * sb);
        }
        pts[row * dp + k] = x;
        s = fmaf(x, x, s);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) sq[row] = s;
}

// u[j*rc + c] = col_scale[j] * col_h[j] * V[j*ldv + c0 + c] for j < nk, 0 for nk <= j < nk_pad.
__global__ void rhs_f32_kernel(const void* __restrict__ V, int v_dtype, int64_t nk, int64_t nk_pad,
                               int ldv, int c0, int rc, const float* __restrict__ cs,
                               const float* __restrict__ ch, float* __restrict__ u) {
    const int64_t total = nk_pad * rc;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = e / rc;
        const int c = (int)(e % rc);
        float val = 0.f;
        if (j < nk) {
            double x = V ? load_as_f64(V, v_dtype, j * ldv + c0 + c) : 1.0;
            if (cs) x *= (double)cs[j];
            if (ch) x *= (double)ch[j];
            val = (float)x;
        }
        u[e] = val;
    }
}

// Transposed bf16 right-hand side for the P.V tensor-core product:
// ut[c*ld + j] = bf16(col_scale[j] * col_h[j] * V[j*ldv + c0 + c]), zero beyond nk.
__global__ void rhs_bf16t_kernel(const void* __restrict__ V, int v_dtype, int64_t nk, int64_t ld,
                                 int ldv, int c0, int rc, const float* __restrict__ cs,
                                 const float* __restrict__ ch, __nv_bfloat16* __restrict__ ut) {
    const int64_t total = ld * rc;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = e / ld, j = e % ld;
        float val = 0.f;
        if (j < nk) {
            double x = V ? load_as_f64(V, v_dtype, j * ldv + c0 + c) : 1.0;
            if (cs) x *= (double)cs[j];
            if (ch) x *= (double)ch[j];
            val = (float)x;
        }
        ut[e] = __float2bfloat16(val);
    }
}

// Per-column maximum of |col_scale_j col_h_j V[j*ldv + c0 + c]| over j, as the
// bit pattern of a non-negative float (so integer atomicMax orders it).
__global__ void rhs_colmax_kernel(const void* __restrict__ V, int v_dtype, int64_t nk, int ldv, int c0, int rc,
                                  const float* __restrict__ cs, const float* __restrict__ ch,
                                  unsigned* __restrict__ colmax) {
    __shared__ unsigned smax[64];
    for (int c = threadIdx.x; c < rc; c += blockDim.x) smax[c] = 0u;
    __syncthreads();
    const int64_t total = nk * rc;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = e / rc;
        const int c = (int)(e % rc);
        double x = V ? load_as_f64(V, v_dtype, j * ldv + c0 + c) : 1.0;
        if (cs) x *= (double)cs[j];
        if (ch) x *= (double)ch[j];
        atomicMax(&smax[c], __float_as_uint(fabsf((float)x)));
    }
    __syncthreads();
    for (int c = threadIdx.x; c < rc; c += blockDim.x) atomicMax(&colmax[c], smax[c]);
}

// Transposed fp16 hi/lo right-hand side with a power-of-two scale per column:
// with x = u_jc / 2^k_c, ut[c*ld + j] = fp16(x) and ut[(rp + c)*ld + j] =
// fp16(x - fp16(x)); colscale[c] = 2^k_c with max_j |u_jc| / 2^k_c in [1/2, 1).
// Rows rc..rp-1 (of both halves) and columns nk..ld-1 are zero.
__global__ void rhs_f16t_kernel(const void* __restrict__ V, int v_dtype, int64_t nk, int64_t ld, int ldv, int c0,
                                int rc, int rp, const float* __restrict__ cs, const float* __restrict__ ch,
                                const unsigned* __restrict__ colmax, __half* __restrict__ ut,
                                float* __restrict__ colscale) {
    if (blockIdx.x == 0)
        for (int c = threadIdx.x; c < rp; c += blockDim.x) {
            int k = 0;
            const float m = c < rc ? __uint_as_float(colmax[c]) : 0.f;
            if (m > 0.f) frexpf(m, &k);
            colscale[c] = ldexpf(1.0f, k);
        }
    const int64_t total = ld * rp;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(e / ld);
        const int64_t j = e - (int64_t)c * ld;
        float val = 0.f;
        if (c < rc && j < nk) {
            double x = V ? load_as_f64(V, v_dtype, j * ldv + c0 + c) : 1.0;
            if (cs) x *= (double)cs[j];
            if (ch) x *= (double)ch[j];
            int k = 0;
            const float m = __uint_as_float(colmax[c]);
            if (m > 0.f) frexpf(m, &k);
            val = (float)ldexp(x, -k);
        }
        const __half hi = __float2half_rn(val);
        ut[e] = hi;
        ut[e + ld * rp] = __float2half_rn(val - __half2float(hi));
    }
}

__global__ void dmap_weights_kernel(const float* __restrict__ D, int64_t n, float alpha,
                                    float* __restrict__ w) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        w[i] = (float)pow((double)D[i], -(double)alpha);
}

__global__ void dmap_rscale_kernel(const float* __restrict__ Kw, const float* __restrict__ w,
                                   int64_t n, float* __restrict__ Da, float* __restrict__ rs) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const double da = (double)Kw[i] * (double)w[i];
        if (Da) Da[i] = (float)da;
        rs[i] = (float)(rsqrt(da) * (double)w[i]);
    }
}

// ---- host launchers --------------------------------------------------------

static int grid_for(int64_t n, int per_block) { return (int)cdiv(n, per_block); }

int launch_sq_norms(const void* X, int dtype, int64_t n, int d, float* sq, cudaStream_t s) {
    if (n == 0) return FD_OK;
    sq_norms_kernel<<<grid_for(n, 8), 256, 0, s>>>(X, dtype, n, d, sq);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

int launch_mean_rows(const void* X, int dtype, int64_t n, int d, float* shift, cudaStream_t s) {
    if (n == 0) {
        FD_CUDA_TRY(cudaMemsetAsync(shift, 0, sizeof(float) * d, s));
        return FD_OK;
    }
    const int64_t cap = 4096;
    const int64_t stride = n > cap ? n / cap : 1;
    const int64_t cnt = n > cap ? cap : n;
    mean_rows_kernel<<<1, 256, 0, s>>>(X, dtype, n, d, stride, cnt, shift);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

int launch_pack(const void* X, int dtype, int64_t n, int d, const float* shift, float beta, int side,
                int tile, void* op, cudaStream_t s) {
    if (n == 0) return FD_OK;
    if (tile == FD_TILE_F16X3) {
        const double sc = sqrt(2.0 * (double)beta * 1.4426950408889634);
        int* status = nullptr;
        FD_TRY(status_word(&status));
        pack_f16x3_kernel<<<grid_for(n, 8), 256, 0, s>>>(X, dtype, n, d, shift, sc, side, kd_f16x3(d), (__half*)op,
                                                         status);
    } else if (tile == FD_TILE_BF16 || tile == FD_TILE_F16) {
        const double sc = sqrt(2.0 * (double)beta * 1.4426950408889634);  // sqrt(2 beta log2(e))
        int* status = nullptr;
        FD_TRY(status_word(&status));
        if (tile == FD_TILE_F16)
            pack16_kernel<H16><<<grid_for(n, 8), 256, 0, s>>>(X, dtype, n, d, shift, sc, side, kd_bf16(d),
                                                             (__half*)op, status);
        else
            pack16_kernel<B16><<<grid_for(n, 8), 256, 0, s>>>(X, dtype, n, d, shift, sc, side, kd_bf16(d),
                                                             (__nv_bfloat16*)op, status);
    } else {
        const int dp = dp_f32(d);
        float* pts = (float*)op;
        float* sq = (float*)((char*)op + align256(sizeof(float) * (size_t)n * dp));
        pack_f32_kernel<<<grid_for(n, 8), 256, 0, s>>>(X, dtype, n, d, shift, sqrt((double)beta), dp,
                                                      pts, sq);
    }
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

int launch_rhs_f32(const void* V, int v_dtype, int64_t nk, int64_t nk_pad, int ldv, int c0, int rc,
                   const float* cs, const float* ch, float* u, cudaStream_t s) {
    const int64_t total = nk_pad * rc;
    if (total == 0) return FD_OK;
    const int grid = (int)std::min<int64_t>(cdiv(total, 256), 148 * 16);
    rhs_f32_kernel<<<grid, 256, 0, s>>>(V, v_dtype, nk, nk_pad, ldv, c0, rc, cs, ch, u);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

int launch_rhs_bf16t(const void* V, int v_dtype, int64_t nk, int64_t ld, int ldv, int c0, int rc,
                     const float* cs, const float* ch, __nv_bfloat16* ut, cudaStream_t s) {
    const int64_t total = ld * rc;
    if (total == 0) return FD_OK;
    const int grid = (int)std::min<int64_t>(cdiv(total, 256), 148 * 16);
    rhs_bf16t_kernel<<<grid, 256, 0, s>>>(V, v_dtype, nk, ld, ldv, c0, rc, cs, ch, ut);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

int launch_rhs_f16t(const void* V, int v_dtype, int64_t nk, int64_t ld, int ldv, int c0, int rc, int rp,
                    const float* cs, const float* ch, unsigned* colmax, __half* ut, float* colscale, cudaStream_t s) {
    FD_CUDA_TRY(cudaMemsetAsync(colmax, 0, sizeof(unsigned) * rp, s));
    if (nk > 0) {
        const int g1 = (int)std::min<int64_t>(cdiv(nk * rc, 256), 148 * 4);
        rhs_colmax_kernel<<<g1, 256, 0, s>>>(V, v_dtype, nk, ldv, c0, rc, cs, ch, colmax);
        FD_CUDA_TRY(cudaGetLastError());
    }
    const int g2 = (int)std::min<int64_t>(cdiv(ld * rp, 256), 148 * 16);
    rhs_f16t_kernel<<<g2, 256, 0, s>>>(V, v_dtype, nk, ld, ldv, c0, rc, rp, cs, ch, colmax, ut, colscale);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

int launch_dmap_weights(const float* D, int64_t n, float alpha, float* w, cudaStream_t s) {
    if (n == 0) return FD_OK;
    dmap_weights_kernel<<<(int)std::min<int64_t>(cdiv(n, 256), 148 * 8), 256, 0, s>>>(D, n, alpha, w);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

int launch_dmap_rscale(const float* Kw, const float* w, int64_t n, float* Da, float* rs, cudaStream_t s) {
    if (n == 0) return FD_OK;
    dmap_rscale_kernel<<<(int)std::min<int64_t>(cdiv(n, 256), 148 * 8), 256, 0, s>>>(Kw, w, n, Da, rs);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

}  // namespace fd
