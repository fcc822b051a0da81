// k nearest squared distances on the tensor cores (the self-tuning bandwidth
// of FD/utils.py:31-52, whose host version sorts a dense N x N matrix).
//
// Two stages:
//   1. screening (knn_tc_kernel): the fp32-class split operands of the
//      operator (FD_TILE_F16X3, one MMA element = -c ||a_q - a_k||^2 to about
//      2^-22 of ||a||^2) give every (query, key) pair a screening score on the
//      tensor cores; each query row keeps its C best keys (C = k + 8 or more)
//      in registers, per key split.
//   2. refinement (knn_refine_kernel): the squared distances of those
//      candidates recomputed exactly as the CUDA-core kernel computes them
//      (fp32 coordinate differences, same summation order), and the k
//      smallest written in ascending order.
// The screening error is four orders of magnitude below the gaps that
// separate the k-th neighbour from the (k + 8)-th on any but degenerate data,
// and ties (duplicated points) are all kept as long as they fit in C.
//
// knn_tc_kernel: one CTA per (128-row query tile, key split); warps 0-3 are
// the epilogue (thread = query row, TMEM lane), warp 4 the TMA producer (query
// tile once, key tiles through a 3-stage ring, no multicast), warp 5 the MMA
// issuer (tcgen05.mma kind::f16, M = 128, N = 128, two TMEM S buffers).
#include <cfloat>
#include <cstring>

#include "fd_tc_common.cuh"

namespace fd {
namespace knn {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int NBUF = 2;
constexpr int TMA_WARP = 4;
constexpr int MMA_WARP = 5;
constexpr int NTHREADS = 6 * 32;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;

template <int KF, int NW>
struct Cfg {
    using G = tc::Geo<KF, NW>;
    static constexpr uint32_t Q_BYTES = G::bytes(BM);
    static constexpr uint32_t STAGE_BYTES = G::bytes(BN);
    static constexpr int STAGES = (int)((220u * 1024u - Q_BYTES) / STAGE_BYTES) > 4
                                      ? 4 : (int)((220u * 1024u - Q_BYTES) / STAGE_BYTES);
    static constexpr uint32_t BAR_OFF = Q_BYTES + STAGES * STAGE_BYTES;
    static constexpr uint32_t MISC_OFF = BAR_OFF + (2 * STAGES + 1 + 2 * NBUF + 1) * 8;
    static constexpr uint32_t SMEM_ALLOC = MISC_OFF + 16 + 1024;
    static_assert(STAGES >= 2, "shared memory budget");
    static_assert(SMEM_ALLOC <= 227 * 1024, "shared memory budget");
};

// Insert (x, j) into the C best scores (descending) of this thread.
template <int C>
__device__ __forceinline__ void keep_best(float (&v)[C], int (&ix)[C], float x, int j) {
#pragma unroll
    for (int s = 0; s < C; ++s) {
        const bool gt = x > v[s];
        const float tv = v[s];
        const int ti = ix[s];
        v[s] = gt ? x : tv;
        ix[s] = gt ? j : ti;
        x = gt ? tv : x;
        j = gt ? ti : j;
    }
}

// Screen 32 scores (keys key0 + col0 .. + 31; columns >= valid are past the
// last key and ignored).  A bit mask of the scores that beat this thread's
// C-th best is formed with constant register indices; the rare scores that
// qualify are then fetched again from TMEM one column at a time (a warp-uniform
// column, the union of the lanes' masks), so no register array is ever
// indexed dynamically (which would move it to local memory).
template <int C>
__device__ __forceinline__ void screen32(const uint32_t (&v)[32], uint32_t tcol, int col0, int64_t key0, int valid,
                                         float (&best)[C], int (&bix)[C]) {
    const float thr = best[C - 1];
    uint32_t mask = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i)
        mask |= (__uint_as_float(v[i]) > thr && col0 + i < valid) ? (1u << i) : 0u;
    uint32_t any = __reduce_or_sync(0xffffffffu, mask);
    while (any) {
        const int i = __ffs(any) - 1;
        any &= any - 1;
        uint32_t x;
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(x) : "r"(tcol + (uint32_t)i) : "memory");
        asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(x) :: "memory");
        const float xf = __uint_as_float(x);
        if (((mask >> i) & 1u) && xf > best[C - 1]) keep_best<C>(best, bix, xf, (int)(key0 + col0 + i));
    }
}

template <int KF, int NW, int C>
__global__ void __launch_bounds__(NTHREADS, 1)
knn_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
              const __grid_constant__ CUtensorMap tmq_n, const __grid_constant__ CUtensorMap tmk_n, int64_t nq,
              int64_t nk, int nsplit, int64_t tiles_per_split, uint32_t idesc, int* __restrict__ cand,
              int* status) {
    using Cf = Cfg<KF, NW>;
    using G = typename Cf::G;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sQ = base;
    uint8_t* sK = base + Cf::Q_BYTES;
    uint64_t* bars = (uint64_t*)(base + Cf::BAR_OFF);
    uint64_t* kfull = bars;
    uint64_t* kempty = kfull + Cf::STAGES;
    uint64_t* qfull = kempty + Cf::STAGES;
    uint64_t* sfull = qfull + 1;
    uint64_t* sempty = sfull + NBUF;
    uint64_t* done = sempty + NBUF;
    uint32_t* tmem_slot = (uint32_t*)(base + Cf::MISC_OFF);
    volatile int* abort = (volatile int*)(base + Cf::MISC_OFF + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t rt = blockIdx.x / nsplit;
    const int sp = (int)(blockIdx.x % nsplit);
    const int64_t n_jt = (nk + BN - 1) / BN;
    const int64_t jt0 = sp * tiles_per_split;
    const int64_t jt1 = jt0 + tiles_per_split < n_jt ? jt0 + tiles_per_split : n_jt;

    if (threadIdx.x == 0) {
        for (int i = 0; i < Cf::STAGES; ++i) {
            ptx::mbar_init(&kfull[i], 1);
            ptx::mbar_init(&kempty[i], 1);
        }
        ptx::mbar_init(qfull, 1);
        for (int i = 0; i < NBUF; ++i) {
            ptx::mbar_init(&sfull[i], 1);
            ptx::mbar_init(&sempty[i], 4);   // the 4 epilogue warps
        }
        ptx::mbar_init(done, 1);
        *abort = 0;
        ptx::fence_mbar_init();
    }
    if (warp == MMA_WARP) {
        ptx::tmem_alloc(tmem_slot, NBUF * BN);
        ptx::tmem_relinquish();
    }
    if (warp == TMA_WARP && lane == 0) {
        ptx::prefetch_tmap(&tmq);
        ptx::prefetch_tmap(&tmk);
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == TMA_WARP) {
        if (lane == 0) {
            ptx::mbar_expect_tx(qfull, Cf::Q_BYTES);
            for (int kb = 0; kb < KF; ++kb) ptx::tma_load_2d(sQ + kb * BM * 128, &tmq, qfull, kb * 64, (int)(rt * BM));
            if (NW) ptx::tma_load_2d(sQ + KF * BM * 128, &tmq_n, qfull, KF * 64, (int)(rt * BM));
            int stage = 0;
            uint32_t kph = 0;
            for (int64_t jt = jt0; jt < jt1; ++jt) {
                if (!ptx::wait_bounded(&kempty[stage], kph ^ 1, abort, status, WAIT_LIMIT_NS)) break;
                uint8_t* st = sK + stage * Cf::STAGE_BYTES;
                ptx::mbar_expect_tx(&kfull[stage], Cf::STAGE_BYTES);
                for (int kb = 0; kb < KF; ++kb) ptx::tma_load_2d(st + kb * BN * 128, &tmk, &kfull[stage], kb * 64, (int)(jt * BN));
                if (NW) ptx::tma_load_2d(st + KF * BN * 128, &tmk_n, &kfull[stage], KF * 64, (int)(jt * BN));
                if (++stage == Cf::STAGES) { stage = 0; kph ^= 1; }
            }
        }
    } else if (warp == MMA_WARP) {
        if (lane == 0) {
            const uint32_t q_base = ptx::smem_u32(sQ), k_base = ptx::smem_u32(sK);
            int stage = 0;
            uint32_t kph = 0;
            if (ptx::wait_bounded(qfull, 0, abort, status, WAIT_LIMIT_NS)) {
                for (int64_t t = 0; t < jt1 - jt0; ++t) {
                    const int b = (int)(t & 1);
                    if (!ptx::wait_bounded(&sempty[b], (uint32_t)(((t >> 1) & 1) ^ 1), abort, status, WAIT_LIMIT_NS)) break;
                    if (!ptx::wait_bounded(&kfull[stage], kph, abort, status, WAIT_LIMIT_NS)) break;
                    ptx::tc_fence_after();
                    const uint32_t ka = k_base + stage * Cf::STAGE_BYTES;
#pragma unroll
                    for (int ks = 0; ks < G::KSTEPS; ++ks)
                        ptx::umma_ss(tmem + b * BN, G::desc(q_base, BM, ks), G::desc(ka, BN, ks), idesc, ks > 0);
                    ptx::umma_commit(&sfull[b]);
                    ptx::umma_commit(&kempty[stage]);
                    if (++stage == Cf::STAGES) { stage = 0; kph ^= 1; }
                }
            }
            ptx::umma_commit(done);
            ptx::wait_bounded(done, 0, abort, status, WAIT_LIMIT_NS);
        }
    } else {
        // epilogue: thread = query row rt * BM + row, its C best keys so far
        const int row = warp * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(warp * 32) << 16);
        float best[C];
        int bix[C];
#pragma unroll
        for (int s = 0; s < C; ++s) { best[s] = -FLT_MAX; bix[s] = -1; }
        for (int64_t t = 0; t < jt1 - jt0; ++t) {
            const int b = (int)(t & 1);
            if (!ptx::wait_bounded(&sfull[b], (uint32_t)((t >> 1) & 1), abort, status, WAIT_LIMIT_NS)) break;
            ptx::tc_fence_after();
            const int64_t key0 = (jt0 + t) * BN;
            const int valid = (int)(nk - key0 < BN ? nk - key0 : BN);   // keys past nk read zero rows
            // four 32-column loads, the next in flight while this one is
            // screened
            uint32_t va[32], vb[32];
            const uint32_t tb = t_lane + b * BN;
            ptx::tmem_ld32(tb, va);
            ptx::tmem_wait_ld(va);
            ptx::tmem_ld32(tb + 32, vb);
            screen32<C>(va, tb, 0, key0, valid, best, bix);
            ptx::tmem_wait_ld(vb);
            ptx::tmem_ld32(tb + 64, va);
            screen32<C>(vb, tb + 32, 32, key0, valid, best, bix);
            ptx::tmem_wait_ld(va);
            ptx::tmem_ld32(tb + 96, vb);
            screen32<C>(va, tb + 64, 64, key0, valid, best, bix);
            ptx::tmem_wait_ld(vb);
            screen32<C>(vb, tb + 96, 96, key0, valid, best, bix);
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&sempty[b]);
        }
        const int64_t gi = rt * BM + row;
        if (gi < nq) {
            int* dst = cand + ((int64_t)gi * nsplit + sp) * C;
#pragma unroll
            for (int s = 0; s < C; ++s) dst[s] = bix[s];
        }
        ptx::tc_fence_before();
    }
    __syncthreads();
    if (warp == MMA_WARP) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, NBUF * BN);
    }
}

// Exact squared distances of the candidates (fp32 coordinate differences
// summed in coordinate order, as the CUDA-core kernel sums them) and the k
// smallest, ascending.  One warp per query row.
__global__ void knn_refine_kernel(const float* __restrict__ Q, int64_t nq, const float* __restrict__ K, int d,
                                  const int* __restrict__ cand, int ncand, int k, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (i >= nq) return;
    const float* q = Q + i * (int64_t)d;
    const int* ci = cand + i * (int64_t)ncand;
    // each lane holds up to 8 candidates (ncand <= 256)
    float dv[8];
    int dj[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int c = lane + 32 * u;
        const int j = c < ncand ? ci[c] : -1;
        float acc = FLT_MAX;
        if (j >= 0) {
            const float* kr = K + (int64_t)j * d;
            acc = 0.f;
            for (int e = 0; e < d; ++e) {
                const float t = q[e] - kr[e];
                acc = fmaf(t, t, acc);
            }
        }
        dv[u] = acc;
        dj[u] = j;
    }
    // k rounds of a warp-wide minimum (ties broken by key index)
    for (int r = 0; r < k; ++r) {
        float m = FLT_MAX;
        int mj = 0x7fffffff, mu = -1;
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (dj[u] >= 0 && (dv[u] < m || (dv[u] == m && dj[u] < mj))) { m = dv[u]; mj = dj[u]; mu = u; }
        float wm = m;
        int wj = mj;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float om = __shfl_xor_sync(0xffffffffu, wm, o);
            const int oj = __shfl_xor_sync(0xffffffffu, wj, o);
            if (om < wm || (om == wm && oj < wj)) { wm = om; wj = oj; }
        }
        if (lane == 0) out[i * (int64_t)k + r] = wm;
        if (mu >= 0 && mj == wj && m == wm) {
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (u == mu) dj[u] = -1;
        }
    }
}

// max over rows of ||x - shift||^2 (as an unsigned bit pattern: non-negative floats order like their bits)
__global__ void max_sqnorm_kernel(const float* __restrict__ X, int64_t n, int d, const float* __restrict__ shift,
                                  unsigned* __restrict__ out) {
    float m = 0.f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float a = 0.f;
        for (int e = 0; e < d; ++e) {
            const float t = X[i * d + e] - shift[e];
            a = fmaf(t, t, a);
        }
        m = fmaxf(m, a);
    }
    atomicMax(out, __float_as_uint(m));
}

struct Plan {
    int kd, kf, nw, C, nsplit;
    int64_t n_rt, n_jt, tiles_per_split;
    size_t off_shift, off_max, off_q, off_k, off_cand, total;
};

static bool plan(int64_t nq, int64_t nk, int d, int k, Plan* p) {
    if (d < 1 || d > 66 || k < 1 || k > 24 || nq < 1 || nk < 1) return false;
    p->kd = kd_f16x3(d);
    split_kd(p->kd, &p->kf, &p->nw);
    p->C = k <= 8 ? 16 : 32;
    p->n_rt = cdiv(nq, BM);
    p->n_jt = cdiv(nk, BN);
    // key splits so that the grid covers the SMs about twice (each split keeps its own C best)
    int ns = (int)cdiv(2 * 148, p->n_rt);
    if (ns > 8) ns = 8;
    if (ns > p->n_jt) ns = (int)p->n_jt;
    if (ns < 1) ns = 1;
    p->tiles_per_split = cdiv(p->n_jt, ns);
    p->nsplit = (int)cdiv(p->n_jt, p->tiles_per_split);
    p->off_shift = 0;
    p->off_max = align256(sizeof(float) * d);
    p->off_q = p->off_max + 256;
    p->off_k = p->off_q + align256((size_t)2 * nq * p->kd);
    p->off_cand = p->off_k + align256((size_t)2 * nk * p->kd);
    p->total = p->off_cand + align256(sizeof(int) * (size_t)nq * p->nsplit * p->C);
    return true;
}

template <int KF, int NW, int C>
static int launch_screen(const Plan& p, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mqn,
                         const CUtensorMap& mkn, int64_t nq, int64_t nk, int* cand, cudaStream_t s) {
    using Cf = Cfg<KF, NW>;
    int* status = nullptr;
    FD_TRY(status_word(&status));
    FD_CUDA_TRY(cudaFuncSetAttribute(knn_tc_kernel<KF, NW, C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)Cf::SMEM_ALLOC));
    knn_tc_kernel<KF, NW, C><<<(unsigned)(p.n_rt * p.nsplit), NTHREADS, Cf::SMEM_ALLOC, s>>>(
        mq, mk, mqn, mkn, nq, nk, p.nsplit, p.tiles_per_split, ptx::idesc_f32acc(BM, BN, true), cand, status);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

template <int KF, int NW>
static int launch_screen_c(const Plan& p, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mqn,
                           const CUtensorMap& mkn, int64_t nq, int64_t nk, int* cand, cudaStream_t s) {
    return p.C == 16 ? launch_screen<KF, NW, 16>(p, mq, mk, mqn, mkn, nq, nk, cand, s)
                     : launch_screen<KF, NW, 32>(p, mq, mk, mqn, mkn, nq, nk, cand, s);
}

}  // namespace knn
}  // namespace fd

using namespace fd;

extern "C" size_t fd_knn_tc_workspace_bytes(int64_t nq, int64_t nk, int d, int k) {
    knn::Plan p;
    return knn::plan(nq, nk, d, k, &p) ? p.total : 0;
}

extern "C" int fd_knn_sqdist_tc(const float* Q, int64_t nq, const float* K, int64_t nk, int d, int k, float* out,
                                void* workspace, size_t workspace_bytes, void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    FD_CHECK_ARG(nq >= 0 && nk >= 0, "fd_knn_sqdist_tc: negative size");
    FD_CHECK_ARG(d >= 1 && d <= 66, "fd_knn_sqdist_tc: d = %d (1..66; fd_knn_sqdist covers larger d)", d);
    FD_CHECK_ARG(k >= 1 && k <= 24, "fd_knn_sqdist_tc: k = %d (1..24; fd_knn_sqdist covers larger k)", k);
    FD_CHECK_ARG(k <= nk, "fd_knn_sqdist_tc: k = %d > %lld keys", k, (long long)nk);
    if (nq == 0) return FD_OK;
    FD_CHECK_ARG(Q && K && out, "fd_knn_sqdist_tc: null pointer");
    knn::Plan p;
    knn::plan(nq, nk, d, k, &p);
    if (workspace_bytes < p.total)
        return set_error(FD_ERR_WORKSPACE, "fd_knn_sqdist_tc: workspace %zu B < required %zu B", workspace_bytes,
                         p.total);
    FD_CHECK_ARG(workspace && ((uintptr_t)workspace & 255) == 0, "workspace must be non-null and 256-byte aligned");
    uint8_t* ws = (uint8_t*)workspace;
    float* shift = (float*)(ws + p.off_shift);
    unsigned* mx = (unsigned*)(ws + p.off_max);
    void* qop = ws + p.off_q;
    void* kop = ws + p.off_k;
    int* cand = (int*)(ws + p.off_cand);
    // common translation, then a scale that keeps every packed value well inside
    // the fp16 range: the screening only ranks, so any positive beta serves
    FD_TRY(launch_mean_rows(K, FD_DTYPE_F32, nk, d, shift, s));
    FD_CUDA_TRY(cudaMemsetAsync(mx, 0, sizeof(unsigned), s));
    knn::max_sqnorm_kernel<<<296, 256, 0, s>>>(K, nk, d, shift, mx);
    knn::max_sqnorm_kernel<<<296, 256, 0, s>>>(Q, nq, d, shift, mx);
    FD_CUDA_TRY(cudaGetLastError());
    unsigned mbits = 0;
    FD_CUDA_TRY(cudaMemcpyAsync(&mbits, mx, sizeof(unsigned), cudaMemcpyDeviceToHost, s));
    FD_CUDA_TRY(cudaStreamSynchronize(s));
    float m;
    memcpy(&m, &mbits, sizeof(m));
    // 2 beta log2(e) max||a||^2 = 4096: packed squared norms of at most 2048
    const float beta = m > 0.f ? (float)(4096.0 / (2.0 * 1.4426950408889634 * (double)m)) : 1.0f;
    FD_TRY(launch_pack(Q, FD_DTYPE_F32, nq, d, shift, beta, FD_SIDE_QUERY, FD_TILE_F16X3, qop, s));
    FD_TRY(launch_pack(K, FD_DTYPE_F32, nk, d, shift, beta, FD_SIDE_KEY, FD_TILE_F16X3, kop, s));
    CUtensorMap mq, mk, mqn, mkn;
    FD_TRY(make_tile_map(&mq, qop, nq, p.kd, knn::BM, true));
    FD_TRY(make_tile_map(&mk, kop, nk, p.kd, knn::BN, true));
    mqn = mq;
    mkn = mk;
    if (p.nw) {
        FD_TRY(make_tile_map(&mqn, qop, nq, p.kd, knn::BM, true, p.nw));
        FD_TRY(make_tile_map(&mkn, kop, nk, p.kd, knn::BN, true, p.nw));
    }
    switch (p.kf * 100 + p.nw) {
        case 16: FD_TRY((knn::launch_screen_c<0, 16>(p, mq, mk, mqn, mkn, nq, nk, cand, s))); break;
        case 32: FD_TRY((knn::launch_screen_c<0, 32>(p, mq, mk, mqn, mkn, nq, nk, cand, s))); break;
        case 100: FD_TRY((knn::launch_screen_c<1, 0>(p, mq, mk, mqn, mkn, nq, nk, cand, s))); break;
        case 116: FD_TRY((knn::launch_screen_c<1, 16>(p, mq, mk, mqn, mkn, nq, nk, cand, s))); break;
        case 132: FD_TRY((knn::launch_screen_c<1, 32>(p, mq, mk, mqn, mkn, nq, nk, cand, s))); break;
        case 200: FD_TRY((knn::launch_screen_c<2, 0>(p, mq, mk, mqn, mkn, nq, nk, cand, s))); break;
        case 216: FD_TRY((knn::launch_screen_c<2, 16>(p, mq, mk, mqn, mkn, nq, nk, cand, s))); break;
        case 232: FD_TRY((knn::launch_screen_c<2, 32>(p, mq, mk, mqn, mkn, nq, nk, cand, s))); break;
        case 300: FD_TRY((knn::launch_screen_c<3, 0>(p, mq, mk, mqn, mkn, nq, nk, cand, s))); break;
        case 316: FD_TRY((knn::launch_screen_c<3, 16>(p, mq, mk, mqn, mkn, nq, nk, cand, s))); break;
        default: return set_error(FD_ERR_UNSUPPORTED, "fd_knn_sqdist_tc: no kernel for kd=%d", p.kd);
    }
    const int ncand = p.nsplit * p.C;
    if (ncand > 256) return set_error(FD_ERR_UNSUPPORTED, "fd_knn_sqdist_tc: %d candidates per row (max 256)", ncand);
    knn::knn_refine_kernel<<<(unsigned)cdiv(nq, 8), 256, 0, s>>>(Q, nq, K, d, cand, ncand, k, out);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}
