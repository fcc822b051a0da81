// fp32-tile path (FD_TILE_F32): CUDA-core SIMT tiles with fp32 distances,
// fp32 exp and fp64 accumulation across key tiles.  Accuracy class of the
// reference NumPy primitive (fp32 GEMM for the cross term, FD/kernel.py:125-134),
// used for the fp32 stage of the eigensolver precision ramp and for shapes the
// tensor-core path does not cover.
//
// Tile: 64 query rows x 64 key columns per block step, 256 threads, each thread
// owning a 4x4 patch of the distance tile.  Operands are staged transposed in
// shared memory ([k][row]) so that a thread reads its 4 rows / 4 columns as
// one float4.  Key tiles are split across gridDim.y when there are too few
// row tiles to fill the GPU; split partials go to an fp64 workspace and are
// summed in a fixed order by simt_reduce_kernel (deterministic).
#include "fd_prep.cuh"

namespace fd {

namespace {
constexpr int SB = 64;        // rows and columns per tile
constexpr int STHREADS = 256;
constexpr int RMAX_SIMT = 64;  // columns of V per launch

struct SimtSmem {
    // offsets in floats inside dynamic shared memory
    int q, k, u, p, acc, qsq, ksq, total_bytes;
};

__host__ __device__ inline SimtSmem simt_layout(int dp, int rc) {
    SimtSmem L;
    int off = 0;
    L.q = off; off += dp * SB;
    L.k = off; off += dp * SB;
    L.qsq = off; off += SB;
    L.ksq = off; off += SB;
    L.u = off; off += SB * rc;
    L.p = off; off += (rc > 1) ? SB * (SB + 1) : 0;
    off = (off + 1) & ~1;  // 8-byte align the fp64 accumulator
    L.acc = off; off += (rc > 1) ? 2 * SB * rc : 0;
    L.total_bytes = off * 4;
    return L;
}
}  // namespace

__global__ void __launch_bounds__(STHREADS)
simt_kernel(const float* __restrict__ qp, const float* __restrict__ qsq, int64_t nq,
            const float* __restrict__ kp, const float* __restrict__ ksq, int64_t nk, int dp,
            const float* __restrict__ u, int rc, float beta, RowEpilogue ep,
            double* __restrict__ part, int64_t jt_per_split) {
    extern __shared__ float4 smem4[];
    float* sm = (float*)smem4;
    const SimtSmem L = simt_layout(dp, rc);
    float* Qs = sm + L.q;    // [dp][SB]
    float* Ks = sm + L.k;    // [dp][SB]
    float* Us = sm + L.u;    // [SB][rc]
    float* Ps = sm + L.p;    // [SB][SB+1]
    double* Acc = (double*)(sm + L.acc);  // [SB][rc]
    float* Qsq = sm + L.qsq;
    float* Ksq = sm + L.ksq;

    const int tid = threadIdx.x;
    const int ty = tid >> 4, tx = tid & 15;
    const int64_t i0 = (int64_t)blockIdx.x * SB;
    const int64_t n_jt = cdiv(nk, SB);
    const int64_t jt_begin = (int64_t)blockIdx.y * jt_per_split;
    const int64_t jt_end = min(n_jt, jt_begin + jt_per_split);

    for (int e = tid; e < SB * dp; e += STHREADS) {
        const int row = e / dp, k = e % dp;
        const int64_t gi = i0 + row;
        Qs[k * SB + row] = gi < nq ? qp[gi * dp + k] : 0.f;
    }
    for (int e = tid; e < SB; e += STHREADS) Qsq[e] = (i0 + e < nq) ? qsq[i0 + e] : 0.f;
    if (rc > 1)
        for (int e = tid; e < SB * rc; e += STHREADS) Acc[e] = 0.0;
    double accr[4] = {0.0, 0.0, 0.0, 0.0};  // r == 1 row accumulators (valid on tx == 0)

    for (int64_t jt = jt_begin; jt < jt_end; ++jt) {
        const int64_t j0 = jt * SB;
        __syncthreads();
        for (int e = tid; e < SB * dp; e += STHREADS) {
            const int col = e / dp, k = e % dp;
            const int64_t gj = j0 + col;
            Ks[k * SB + col] = gj < nk ? kp[gj * dp + k] : 0.f;
        }
        for (int e = tid; e < SB; e += STHREADS) Ksq[e] = (j0 + e < nk) ? ksq[j0 + e] : 0.f;
        for (int e = tid; e < SB * rc; e += STHREADS) Us[e] = u[j0 * rc + e];  // u is zero-padded
        __syncthreads();

        float dot[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) dot[a][b] = 0.f;
        for (int k = 0; k < dp; ++k) {
            const float4 qa = *(const float4*)&Qs[k * SB + ty * 4];
            const float4 kb = *(const float4*)&Ks[k * SB + tx * 4];
            const float qv[4] = {qa.x, qa.y, qa.z, qa.w};
            const float kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) dot[a][b] = fmaf(qv[a], kv[b], dot[a][b]);
        }
        float p[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int col = tx * 4 + b;
                float d2 = Qsq[ty * 4 + a] + Ksq[col] - 2.0f * dot[a][b];
                d2 = fmaxf(d2, 0.0f);
                p[a][b] = (j0 + col < nk) ? expf(-beta * d2) : 0.f;
            }
        if (rc == 1) {
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                float s = 0.f;
#pragma unroll
                for (int b = 0; b < 4; ++b) s = fmaf(p[a][b], Us[tx * 4 + b], s);
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                accr[a] += (double)s;
            }
        } else {
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) Ps[(ty * 4 + a) * (SB + 1) + tx * 4 + b] = p[a][b];
            __syncthreads();
            for (int e = tid; e < SB * rc; e += STHREADS) {
                const int row = e / rc, c = e % rc;
                float s = 0.f;
#pragma unroll 8
                for (int j = 0; j < SB; ++j) s = fmaf(Ps[row * (SB + 1) + j], Us[j * rc + c], s);
                Acc[e] += (double)s;
            }
        }
    }
    __syncthreads();

    const bool split = gridDim.y > 1;
    if (rc == 1) {
        if (tx == 0) {
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                const int64_t gi = i0 + ty * 4 + a;
                if (gi >= nq) continue;
                if (split) part[(int64_t)blockIdx.y * nq + gi] = accr[a];
                else store_out(ep, gi, 0, accr[a]);
            }
        }
    } else {
        for (int e = tid; e < SB * rc; e += STHREADS) {
            const int row = e / rc, c = e % rc;
            const int64_t gi = i0 + row;
            if (gi >= nq) continue;
            if (split) part[((int64_t)blockIdx.y * nq + gi) * rc + c] = Acc[e];
            else store_out(ep, gi, c, Acc[e]);
        }
    }
}

// ---- r = 1: 128 x 128 tiles, 8 x 8 per thread, cp.async double buffering ------
// Rows ty + 16a and columns tx + 16b of the tile belong to thread (ty, tx):
// operands stay row-major in shared memory with a row pitch dpp = 4 x odd
// floats, so the float4 reads of 16 lanes with consecutive tx hit distinct
// bank groups and the query reads are broadcasts.  The next key tile (points,
// squared norms, u) is copied by cp.async while the current one is computed;
// rows past nk are zero-filled and masked.  One CTA per SM (up to 222 KB of
// shared memory); fp32 dot products, expf, fp32 row sums within a tile, fp64
// across tiles -- the accuracy class of the 64 x 64 kernel above.
namespace {
constexpr int TB = 128;
__host__ __device__ inline int simt1_pitch(int dp) { return ((dp / 4) & 1) ? dp : dp + 4; }
__host__ __device__ inline size_t simt1_smem(int dp) {
    return sizeof(float) * ((size_t)3 * TB * simt1_pitch(dp) + 5 * TB);
}
__device__ __forceinline__ void cp_async(void* dst, const void* src, int bytes, bool valid) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    if (bytes == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(valid ? 16 : 0)
                     : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(valid ? 4 : 0)
                     : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
}  // namespace

__global__ void __launch_bounds__(STHREADS, 1)
simt1_kernel(const float* __restrict__ qp, const float* __restrict__ qsq, int64_t nq,
             const float* __restrict__ kp, const float* __restrict__ ksq, int64_t nk, int dp,
             const float* __restrict__ u, float beta, RowEpilogue ep, double* __restrict__ part,
             int64_t jt_per_split) {
    extern __shared__ float4 smem4[];
    float* sm = (float*)smem4;
    const int dpp = simt1_pitch(dp);
    float* Qs = sm;                          // [TB][dpp]
    float* Ks = Qs + TB * dpp;               // [2][TB][dpp]
    float* Qsq = Ks + 2 * TB * dpp;          // [TB]
    float* Ksq = Qsq + TB;                   // [2][TB]
    float* Us = Ksq + 2 * TB;                // [2][TB]
    const int tid = threadIdx.x;
    const int ty = tid >> 4, tx = tid & 15;
    const int64_t i0 = (int64_t)blockIdx.x * TB;
    const int64_t n_jt = cdiv(nk, TB);
    const int64_t jt_begin = (int64_t)blockIdx.y * jt_per_split;
    const int64_t jt_end = min(n_jt, jt_begin + jt_per_split);
    const int c4n = dp / 4;

    auto load_rows = [&](float* dst, const float* src, int64_t r0, int64_t n) {
        for (int e = tid; e < TB * c4n; e += STHREADS) {
            const int r = e / c4n, c4 = e - r * c4n;
            const int64_t g = r0 + r;
            cp_async(dst + r * dpp + c4 * 4, src + (g < n ? g : 0) * dp + c4 * 4, 16, g < n);
        }
    };
    auto load_keys = [&](int64_t jt, int buf) {
        const int64_t j0 = jt * TB;
        load_rows(Ks + buf * TB * dpp, kp, j0, nk);
        if (tid < TB) {
            const int64_t g = j0 + tid;
            cp_async(Ksq + buf * TB + tid, ksq + (g < nk ? g : 0), 4, g < nk);
            cp_async(Us + buf * TB + tid, u + (g < nk ? g : 0), 4, g < nk);
        }
    };
    load_rows(Qs, qp, i0, nq);
    if (tid < TB) cp_async(Qsq + tid, qsq + (i0 + tid < nq ? i0 + tid : 0), 4, i0 + tid < nq);
    if (jt_begin < jt_end) load_keys(jt_begin, 0);
    cp_async_commit();

    double accr[8];
#pragma unroll
    for (int a = 0; a < 8; ++a) accr[a] = 0.0;
    int buf = 0;
    for (int64_t jt = jt_begin; jt < jt_end; ++jt, buf ^= 1) {
        if (jt + 1 < jt_end) load_keys(jt + 1, buf ^ 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const float* Kb = Ks + buf * TB * dpp;
        float dot[8][8];
#pragma unroll
        for (int a = 0; a < 8; ++a)
#pragma unroll
            for (int b = 0; b < 8; ++b) dot[a][b] = 0.f;
        for (int k = 0; k < dp; k += 4) {
            float4 qv[8], kv[8];
#pragma unroll
            for (int a = 0; a < 8; ++a) qv[a] = *(const float4*)&Qs[(ty + 16 * a) * dpp + k];
#pragma unroll
            for (int b = 0; b < 8; ++b) kv[b] = *(const float4*)&Kb[(tx + 16 * b) * dpp + k];
#pragma unroll
            for (int a = 0; a < 8; ++a)
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    dot[a][b] = fmaf(qv[a].x, kv[b].x, dot[a][b]);
                    dot[a][b] = fmaf(qv[a].y, kv[b].y, dot[a][b]);
                    dot[a][b] = fmaf(qv[a].z, kv[b].z, dot[a][b]);
                    dot[a][b] = fmaf(qv[a].w, kv[b].w, dot[a][b]);
                }
        }
        const int64_t j0 = jt * TB;
        float kq[8], uu[8];
        bool ok[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            kq[b] = Ksq[buf * TB + tx + 16 * b];
            uu[b] = Us[buf * TB + tx + 16 * b];
            ok[b] = j0 + tx + 16 * b < nk;
        }
#pragma unroll
        for (int a = 0; a < 8; ++a) {
            const float qq = Qsq[ty + 16 * a];
            float sa = 0.f;
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const float d2 = fmaxf(qq + kq[b] - 2.0f * dot[a][b], 0.0f);
                const float pv = ok[b] ? expf(-beta * d2) : 0.f;
                sa = fmaf(pv, uu[b], sa);
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) sa += __shfl_xor_sync(0xffffffffu, sa, o);
            accr[a] += (double)sa;
        }
        __syncthreads();   // the next iteration's copies overwrite this buffer pair's other half
    }
    cp_async_wait<0>();
    if (tx == 0) {
        const bool split = gridDim.y > 1;
#pragma unroll
        for (int a = 0; a < 8; ++a) {
            const int64_t gi = i0 + ty + 16 * a;
            if (gi >= nq) continue;
            if (split) part[(int64_t)blockIdx.y * nq + gi] = accr[a];
            else store_out(ep, gi, 0, accr[a]);
        }
    }
}

static bool simt1_ok(int dp, int rc) { return rc == 1 && simt1_smem(dp) <= 227u * 1024u; }

static int simt1_splits(int64_t nq, int64_t nk) {
    const int64_t n_rt = cdiv(nq, TB), n_jt = cdiv(nk, TB);
    const int64_t target = 148 * 2;
    int64_t sp = n_rt >= target ? 1 : cdiv(target, std::max<int64_t>(n_rt, 1));
    sp = std::min<int64_t>(sp, std::max<int64_t>(n_jt, 1));
    return (int)std::min<int64_t>(sp, 64);
}

__global__ void simt_reduce_kernel(const double* __restrict__ part, int nsplit, int64_t nq, int rc,
                                   RowEpilogue ep) {
    const int64_t total = nq * rc;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        double s = 0.0;
        for (int k = 0; k < nsplit; ++k) s += part[(int64_t)k * total + e];
        store_out(ep, e / rc, (int)(e % rc), s);
    }
}

static int simt_splits(int64_t nq, int64_t nk) {
    const int64_t n_rt = cdiv(nq, SB), n_jt = cdiv(nk, SB);
    const int64_t target = 148 * 4;
    int64_t sp = n_rt >= target ? 1 : cdiv(target, std::max<int64_t>(n_rt, 1));
    sp = std::min<int64_t>(sp, std::max<int64_t>(n_jt, 1));
    return (int)std::min<int64_t>(sp, 64);
}

size_t simt_workspace_bytes(int64_t nq, int64_t nk, int rc) {
    const int sp = std::max(simt_splits(nq, nk), rc == 1 ? simt1_splits(nq, nk) : 1);
    return sp > 1 ? align256(sizeof(double) * (size_t)sp * nq * std::min(rc, RMAX_SIMT)) : 0;
}

int launch_simt(const float* qpts, const float* qsq, int64_t nq, const float* kpts, const float* ksq,
                int64_t nk, int d, const float* u, int rc, float beta, const RowEpilogue& ep,
                void* ws, size_t ws_bytes, cudaStream_t s) {
    FD_CHECK_ARG(rc >= 1 && rc <= RMAX_SIMT, "fp32 tile path: %d columns per launch (max %d)", rc, RMAX_SIMT);
    if (nq == 0) return FD_OK;
    const int dp = dp_f32(d);
    if (nk > 0 && simt1_ok(dp, rc)) {
        const size_t smem = simt1_smem(dp);
        FD_CUDA_TRY(cudaFuncSetAttribute(simt1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        const int sp = simt1_splits(nq, nk);
        const int64_t n_jt = cdiv(nk, TB);
        const int64_t per = cdiv(n_jt, sp);
        const int nsp = (int)cdiv(n_jt, per);
        double* part = nullptr;
        if (nsp > 1) {
            const size_t need = sizeof(double) * (size_t)nsp * nq;
            if (ws_bytes < need)
                return set_error(FD_ERR_WORKSPACE, "fp32 tile path: workspace %zu B < %zu B", ws_bytes, need);
            part = (double*)ws;
        }
        dim3 grid((unsigned)cdiv(nq, TB), (unsigned)nsp);
        simt1_kernel<<<grid, STHREADS, smem, s>>>(qpts, qsq, nq, kpts, ksq, nk, dp, u, beta, ep, part, per);
        FD_CUDA_TRY(cudaGetLastError());
        if (nsp > 1) {
            simt_reduce_kernel<<<(int)std::min<int64_t>(cdiv(nq, 256), 148 * 8), 256, 0, s>>>(part, nsp, nq, 1, ep);
            FD_CUDA_TRY(cudaGetLastError());
        }
        return FD_OK;
    }
    const SimtSmem L = simt_layout(dp, rc);
    if (L.total_bytes > 227 * 1024)
        return set_error(FD_ERR_UNSUPPORTED, "fp32 tile path: d=%d r=%d needs %d B of shared memory",
                         d, rc, L.total_bytes);
    FD_CUDA_TRY(cudaFuncSetAttribute(simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     L.total_bytes));
    const int sp = nk == 0 ? 1 : simt_splits(nq, nk);
    const int64_t n_jt = cdiv(nk, SB);
    const int64_t per = sp > 1 ? cdiv(n_jt, sp) : n_jt;
    const int nsp = sp > 1 ? (int)cdiv(n_jt, per) : 1;
    double* part = nullptr;
    if (nsp > 1) {
        const size_t need = sizeof(double) * (size_t)nsp * nq * rc;
        if (ws_bytes < need)
            return set_error(FD_ERR_WORKSPACE, "fp32 tile path: workspace %zu B < %zu B", ws_bytes, need);
        part = (double*)ws;
    }
    dim3 grid((unsigned)cdiv(nq, SB), (unsigned)nsp);
    simt_kernel<<<grid, STHREADS, L.total_bytes, s>>>(qpts, qsq, nq, kpts, ksq, nk, dp, u, rc, beta, ep,
                                                      part, per);
    FD_CUDA_TRY(cudaGetLastError());
    if (nsp > 1) {
        const int64_t total = nq * rc;
        simt_reduce_kernel<<<(int)std::min<int64_t>(cdiv(total, 256), 148 * 8), 256, 0, s>>>(
            part, nsp, nq, rc, ep);
        FD_CUDA_TRY(cudaGetLastError());
    }
    return FD_OK;
}

}  // namespace fd
