// 16-bit tensor-core path (FD_TILE_F16 / FD_TILE_BF16) of the Gaussian-kernel operator on
// sm_100a: a persistent, warp-specialised kernel.
//
//   out_i = ep_i * sum_j 2^( q~_i . k~_j ) * u_j          (q~.k~ <= 0 up to rounding)
//
// The packed operands fold the squared norms and -beta*log2(e) into the dot
// product (layout in fd_common.cuh), so the whole exponent of one (i,j) pair
// is a single tcgen05 MMA accumulator element; the epilogue is
// exp2 (MUFU, or a polynomial on the FMA pipe for a fixed share of the
// columns) -> packed f32x2 FMA with u_j (staged in shared memory by TMA).
//
// CTA = 256 query rows (two 128-row subtiles sharing every key tile) x
// stream of 128-row key tiles.  Warp roles (19 warps):
//   warps 0-15  four epilogue warpgroups (subtile s, parity p): WG(s,p) owns the
//               TMEM S buffer 2s+p and the key tiles of parity p of subtile s
//   warp  16    TMA producer: query tile once per row tile, key tiles through
//               a STAGES-deep shared-memory ring (no multicast), and the
//               matching 128 values of u through a 4-deep ring (bulk copies)
//   warps 17-18 MMA issuers, one per query subtile: tcgen05.mma kind::f16,
//               M=128 N=128 K=16 steps
// Work split: the (row tile, key tile) pairs are cut into gridDim.x contiguous
// ranges (persistent CTAs, one per SM).  A row tile fully inside one range is
// written directly; a row tile cut between ranges leaves fp64 partials in the
// workspace that tc_fixup_kernel sums in CTA order (deterministic).

#include <mutex>

#include "fd_tc_common.cuh"

namespace fd {

__device__ int g_fd_status = 0;

namespace tc {

constexpr int BM = 128;     // rows per subtile = TMEM lanes
constexpr int NSUB = 2;     // subtiles per CTA
constexpr int ROWS = BM * NSUB;
constexpr int BN = 128;     // key rows per tile = S columns
constexpr int TMA_WARP = 16;
constexpr int MMA_WARP = 17;    // MMA issuer of query subtile 0 (and TMEM owner); warp 18 issues subtile 1
constexpr int NTHREADS = 19 * 32;
constexpr uint32_t BOX_BYTES = 128 * 128;  // one 128-row x 64-col 16-bit box (128-byte rows)
constexpr uint32_t TMEM_COLS = 512;
constexpr int URING = 4;                    // depth of the right-hand-side ring
constexpr uint32_t U_BYTES = BN * 4;        // one key tile of u (fp32)
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // 2 s per pipeline wait

template <int KF, int NW>
struct Cfg {
    using G = Geo<KF, NW>;
    static constexpr uint32_t SUB_BYTES = G::bytes(BM);        // one query subtile
    static constexpr uint32_t Q_BYTES = NSUB * SUB_BYTES;
    static constexpr uint32_t STAGE_BYTES = G::bytes(BN);      // one key tile
    static constexpr int STAGES_RAW = (int)((220u * 1024u - Q_BYTES - URING * U_BYTES) / STAGE_BYTES);
    static constexpr int STAGES = STAGES_RAW > 6 ? 6 : STAGES_RAW;
    static_assert(STAGES >= 2, "shared memory budget");
    static constexpr uint32_t U_OFF = Q_BYTES + STAGES * STAGE_BYTES;
    static constexpr uint32_t BAR_OFF = U_OFF + URING * U_BYTES;
    // barriers: kfull[S], kempty[S], ufull[U], uempty[U], qfull, qempty, sfull[4], sempty[4],
    //           rfull[2], rempty[2], done[2]
    static constexpr int NBARS = 2 * STAGES + 2 * URING + 2 + 8 + 4 + 2;
    static constexpr uint32_t MISC_OFF = BAR_OFF + NBARS * 8;
    static constexpr uint32_t RED_OFF = (MISC_OFF + 16 + 15) & ~15u;
    static constexpr uint32_t SMEM_BYTES = RED_OFF + NSUB * BM * 8;
    static constexpr uint32_t SMEM_ALLOC = SMEM_BYTES + 1024;  // slack for 1024-byte alignment
};

// 16 columns of S for r = 1: acc += 2^S . u (column pairs packed).  Columns
// [0, EMU) of the 16 take the FMA-pipe exponential, the rest MUFU.
template <int EMU>
__device__ __forceinline__ void chunk16_r1(const uint32_t (&v)[16], const float* us, uint64_t& acc_a,
                                           uint64_t& acc_b) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint64_t ua, ub;
        ptx::lds_pairs(us + 4 * q, ua, ub);
        const uint64_t e01 = (4 * q + 2 <= EMU) ? exp2_poly2(v[4 * q], v[4 * q + 1])
                                                : exp2_mufu2(v[4 * q], v[4 * q + 1]);
        const uint64_t e23 = (4 * q + 4 <= EMU) ? exp2_poly2(v[4 * q + 2], v[4 * q + 3])
                                                : exp2_mufu2(v[4 * q + 2], v[4 * q + 3]);
        acc_a = ptx::fma2(e01, ua, acc_a);
        acc_b = ptx::fma2(e23, ub, acc_b);
    }
}

template <int KF, int NW, int EMU>
__global__ void __launch_bounds__(NTHREADS, 1)
tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
          const __grid_constant__ CUtensorMap tmq_n, const __grid_constant__ CUtensorMap tmk_n,
          const float* __restrict__ u, int64_t nq, uint32_t idesc, Sched sc, RowEpilogue ep,
          double* __restrict__ part, int* __restrict__ status) {
    using C = Cfg<KF, NW>;
    using G = typename C::G;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sQ = base;
    uint8_t* sK = base + C::Q_BYTES;
    float* sU = (float*)(base + C::U_OFF);
    uint64_t* bars = (uint64_t*)(base + C::BAR_OFF);
    uint64_t* kfull = bars;
    uint64_t* kempty = kfull + C::STAGES;
    uint64_t* ufull = kempty + C::STAGES;
    uint64_t* uempty = ufull + URING;
    uint64_t* qfull = uempty + URING;
    uint64_t* qempty = qfull + 1;
    uint64_t* sfull = qfull + 2;
    uint64_t* sempty = sfull + 4;
    uint64_t* rfull = sempty + 4;
    uint64_t* rempty = rfull + 2;
    uint64_t* done = rempty + 2;
    uint32_t* tmem_slot = (uint32_t*)(base + C::MISC_OFF);
    volatile int* abort = (volatile int*)(base + C::MISC_OFF + 4);
    double* red = (double*)(base + C::RED_OFF);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int cta = blockIdx.x;

    if (threadIdx.x == 0) {
        for (int i = 0; i < C::STAGES; ++i) {
            ptx::mbar_init(&kfull[i], 1);
            ptx::mbar_init(&kempty[i], 2);  // both MMA issuers
        }
        for (int i = 0; i < URING; ++i) {
            ptx::mbar_init(&ufull[i], 1);
            ptx::mbar_init(&uempty[i], 8);  // the 8 epilogue warps of one parity
        }
        ptx::mbar_init(qfull, 1);
        ptx::mbar_init(qempty, 2);          // both MMA issuers
        for (int i = 0; i < 4; ++i) {
            ptx::mbar_init(&sfull[i], 1);
            ptx::mbar_init(&sempty[i], 4);  // one arrive per epilogue warp
        }
        for (int i = 0; i < 2; ++i) {
            ptx::mbar_init(&rfull[i], BM);
            ptx::mbar_init(&rempty[i], BM);
        }
        ptx::mbar_init(&done[0], 1);
        ptx::mbar_init(&done[1], 1);
        *abort = 0;
        ptx::fence_mbar_init();
    }
    if (warp == MMA_WARP) {
        ptx::tmem_alloc(tmem_slot, TMEM_COLS);
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
            int stage = 0;
            uint32_t kph = 0, qcount = 0;
            int64_t cur_rt = -1;
            bool pacing = true;
            int64_t paced = -1;
            for (Walk w(sc, cta); !w.done(); w.next()) {
                const int64_t m = w.s, rt = w.rt, jt = w.jt;
                if (rt != cur_rt) {
                    if (qcount > 0 && !ptx::wait_bounded(qempty, (qcount - 1) & 1, abort, status, WAIT_LIMIT_NS)) break;
                    ptx::mbar_expect_tx(qfull, C::Q_BYTES);
                    for (int s = 0; s < NSUB; ++s) {
                        for (int kb = 0; kb < KF; ++kb)
                            ptx::tma_load_2d(sQ + s * C::SUB_BYTES + kb * BOX_BYTES, &tmq, qfull, kb * 64,
                                             (int)(rt * ROWS + s * BM));
                        if (NW) ptx::tma_load_2d(sQ + s * C::SUB_BYTES + KF * BOX_BYTES, &tmq_n, qfull, KF * 64,
                                                 (int)(rt * ROWS + s * BM));
                    }
                    cur_rt = rt;
                    ++qcount;
                }
                if (pacing) pacing = pace(sc, m, jt, abort, paced);
                if (!ptx::wait_bounded(&kempty[stage], kph ^ 1, abort, status, WAIT_LIMIT_NS)) break;
                ptx::mbar_expect_tx(&kfull[stage], C::STAGE_BYTES);
                for (int kb = 0; kb < KF; ++kb)
                    ptx::tma_load_2d(sK + stage * C::STAGE_BYTES + kb * BOX_BYTES, &tmk, &kfull[stage], kb * 64,
                                     (int)(jt * BN));
                if (NW) ptx::tma_load_2d(sK + stage * C::STAGE_BYTES + KF * BOX_BYTES, &tmk_n, &kfull[stage],
                                         KF * 64, (int)(jt * BN));
                if (++stage == C::STAGES) { stage = 0; kph ^= 1; }
                // right-hand side of this key tile into the u ring
                const int us = (int)(m & (URING - 1));
                const uint32_t uph = (uint32_t)((m / URING) & 1);
                if (!ptx::wait_bounded(&uempty[us], uph ^ 1, abort, status, WAIT_LIMIT_NS)) break;
                ptx::mbar_expect_tx(&ufull[us], U_BYTES);
                ptx::bulk_load(sU + us * BN, u + jt * BN, U_BYTES, &ufull[us]);
            }
        }
    } else if (warp == MMA_WARP || warp == MMA_WARP + 1) {
        // one issuing warp per query subtile: a tcgen05.mma costs its issuing
        // thread about 100 cycles whatever its size, so the two independent
        // Q.K^T chains of a key tile get two issuers
        if (lane == 0) {
            const int s = warp - MMA_WARP;
            const uint32_t q_base = ptx::smem_u32(sQ), k_base = ptx::smem_u32(sK);
            int stage = 0;
            uint32_t kph = 0, qcount = 0;
            int64_t cur_rt = -1;
            for (Walk w(sc, cta); !w.done(); w.next()) {
                const int64_t m = w.s, rt = w.rt;
                const int p = (int)(m & 1);
                const uint32_t use = (uint32_t)(m >> 1);
                if (rt != cur_rt) {
                    if (!ptx::wait_bounded(qfull, qcount & 1, abort, status, WAIT_LIMIT_NS)) break;
                    ++qcount;
                    cur_rt = rt;
                }
                if (!ptx::wait_bounded(&kfull[stage], kph, abort, status, WAIT_LIMIT_NS)) break;
                {
                    const int b = s * 2 + p;
                    if (!ptx::wait_bounded(&sempty[b], (use & 1) ^ 1, abort, status, WAIT_LIMIT_NS)) break;
                    ptx::tc_fence_after();
                    const uint32_t qa = q_base + s * C::SUB_BYTES;
                    const uint32_t ka = k_base + stage * C::STAGE_BYTES;
#pragma unroll
                    for (int ks = 0; ks < G::KSTEPS; ++ks)
                        ptx::umma_ss(tmem + b * BN, G::desc(qa, BM, ks), G::desc(ka, BN, ks), idesc, ks > 0);
                    ptx::umma_commit(&sfull[b]);
                }
                ptx::umma_commit(&kempty[stage]);
                if (w.seg_last()) ptx::umma_commit(qempty);
                if (++stage == C::STAGES) { stage = 0; kph ^= 1; }
            }
            // every MMA issued above has completed once `done` flips
            ptx::umma_commit(&done[s]);
            ptx::wait_bounded(&done[s], 0, abort, status, WAIT_LIMIT_NS);
        }
    } else {
        // ---- epilogue warpgroups ------------------------------------------
        const int wg = warp >> 2;
        const int s = wg >> 1, p = wg & 1;
        const int quarter = warp & 3;
        const int row_in_tile = s * BM + quarter * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
        double acc = 0.0;
        uint32_t segs = 0;
        bool alive = true;
        for (Walk w(sc, cta); !w.done() && alive; w.next()) {
            const int64_t m = w.s, rt = w.rt;
            if ((int)(m & 1) == p) {
                const uint32_t use = (uint32_t)(m >> 1);
                const int b = s * 2 + p;
                const int us = (int)(m & (URING - 1));
                if (!ptx::wait_bounded(&ufull[us], (uint32_t)((m / URING) & 1), abort, status, WAIT_LIMIT_NS)) { alive = false; break; }
                if (!ptx::wait_bounded(&sfull[b], use & 1, abort, status, WAIT_LIMIT_NS)) { alive = false; break; }
                ptx::tc_fence_after();
                const float* ut = sU + us * BN;
                uint64_t acc_a = 0, acc_b = 0;   // +0.0f pairs
                // 16-column TMEM loads, double buffered: the load of the next
                // 16 columns is in flight while the current 16 are computed
                uint32_t va[16], vb[16];
                const uint32_t tb = t_lane + b * BN;
                ptx::tmem_ld16(tb, va);
                ptx::tmem_wait_ld16(va);
#pragma unroll 1
                for (int c = 0; c < BN / 16; c += 2) {
                    ptx::tmem_ld16(tb + (c + 1) * 16, vb);
                    chunk16_r1<EMU>(va, ut + c * 16, acc_a, acc_b);
                    ptx::tmem_wait_ld16(vb);
                    if (c + 2 < BN / 16) ptx::tmem_ld16(tb + (c + 2) * 16, va);
                    chunk16_r1<EMU>(vb, ut + (c + 1) * 16, acc_a, acc_b);
                    if (c + 2 < BN / 16) ptx::tmem_wait_ld16(va);
                }
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    ptx::mbar_arrive(&sempty[b]);
                    ptx::mbar_arrive(&uempty[us]);
                }
                uint32_t a0, a1, b0, b1;
                ptx::unpack2(acc_a, a0, a1);
                ptx::unpack2(acc_b, b0, b1);
                acc += (double)((__uint_as_float(a0) + __uint_as_float(a1)) + (__uint_as_float(b0) + __uint_as_float(b1)));
            }
            if (w.seg_last()) {
                // combine the two parity halves of this subtile, then store
                const uint32_t ph = segs & 1;
                if (p == 1) {
                    if (!ptx::wait_bounded(&rempty[s], ph ^ 1, abort, status, WAIT_LIMIT_NS)) { alive = false; break; }
                    red[s * BM + quarter * 32 + lane] = acc;
                    ptx::mbar_arrive(&rfull[s]);
                } else {
                    if (!ptx::wait_bounded(&rfull[s], ph, abort, status, WAIT_LIMIT_NS)) { alive = false; break; }
                    const double tot = acc + red[s * BM + quarter * 32 + lane];
                    ptx::mbar_arrive(&rempty[s]);
                    const int64_t gi = rt * ROWS + row_in_tile;
                    if (gi < nq) {
                        if (w.seg_full()) store_out(ep, gi, 0, tot);
                        else part[((int64_t)cta * 2 + w.slot()) * ROWS + row_in_tile] = tot;
                    }
                }
                acc = 0.0;
                ++segs;
            }
        }
        ptx::tc_fence_before();
    }
    __syncthreads();
    if (warp == MMA_WARP) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// Sum the partials of row tiles cut between CTA ranges, in CTA order.
__global__ void tc_fixup_kernel(const double* __restrict__ part, Sched sc, int64_t nq, RowEpilogue ep) {
    const int64_t rt = blockIdx.x;
    for (int r = threadIdx.x; r < ROWS; r += blockDim.x) {
        const int64_t gi = rt * ROWS + r;
        if (gi >= nq) continue;
        double sum = 0.0;
        const bool cut = for_each_cut_owner(sc, rt, [&](int c, int slot) {
            sum += part[((int64_t)c * 2 + slot) * ROWS + r];
        });
        if (cut) store_out(ep, gi, 0, sum);
    }
}


// ---- wide operands: kd in (208, 416] -------------------------------------------
// The fp32-class split operands (FD_TILE_F16X3, kd = 3d + 6 rounded) of
// d = 68..136, and 16-bit operands of d > 202, do not fit the kernel above
// (its 256-row query tile plus whole-key-tile stages would need up to 310 KB
// of shared memory).  tcw_kernel keeps a 128-row query tile resident and
// streams each key tile as its 64-column boxes through a ring of 16 KB slots,
// so the Q.K^T chain of a tile waits box by box; four TMEM S buffers (all 512
// columns) let four epilogue warpgroups (tile m -> warpgroup m mod 4) overlap
// the chain.  Two independent producer -> issuer pipelines, one for the even
// and one for the odd tiles, each with its own half of the box ring (a single
// consumer per sub-ring, in order), so the chain of one waits on a box while
// the other's keeps the tensor pipe fed.  Warp roles (20 warps): 0-15 epilogue,
// 16 / 19 TMA producers of the even / odd tiles (16 also loads the query tile
// once per row tile; u through a 4-deep ring), 17 / 18 the MMA issuers of the
// even / odd tiles.  2 kd tensor flops per evaluation.
namespace w {
constexpr int BM = 128;                 // query rows per tile = TMEM lanes
constexpr int BN = 128;                 // keys per tile
constexpr int NSB = 4;                  // S buffers = epilogue warpgroups
constexpr int TMA_WARP = 16;           // producer of the even tiles (and of the query tile)
constexpr int MMA_WARP = 17;           // issuer of the even tiles; 18: odd tiles
constexpr int TMA_WARP_ODD = 19;       // producer of the odd tiles
constexpr int NTHREADS = 20 * 32;
constexpr uint32_t SLOT_BYTES = BN * 128;   // one 64-column box of a key tile

template <int KF, int NW>
struct Cfg {
    static constexpr int NB = KF + (NW ? 1 : 0);                      // boxes per key tile
    static constexpr uint32_t Q_BYTES = BM * (KF * 128 + NW * 2);
    static constexpr uint32_t NARROW_BYTES = BN * NW * 2;
    static constexpr int SLOTS_RAW = (int)((221u * 1024u - Q_BYTES - URING * U_BYTES) / SLOT_BYTES);
    static constexpr int SLOTS = SLOTS_RAW > 12 ? 12 : SLOTS_RAW;
    static_assert(SLOTS >= 4, "shared memory budget");
    static constexpr int SH = SLOTS / 2;                               // slots per pipeline
    static constexpr uint32_t RING_OFF = (Q_BYTES + 1023) & ~1023u;
    static constexpr uint32_t U_OFF = RING_OFF + SLOTS * SLOT_BYTES;
    static constexpr uint32_t BAR_OFF = U_OFF + URING * U_BYTES;
    // kfull[S], kempty[S], ufull[U], uempty[U], qfull, qempty, sfull[4], sempty[4], rfull, rempty, done[2]
    static constexpr int NBARS = 2 * SLOTS + 2 * URING + 2 + 2 * NSB + 4;
    static constexpr uint32_t MISC_OFF = BAR_OFF + NBARS * 8;
    static constexpr uint32_t RED_OFF = (MISC_OFF + 16 + 15) & ~15u;
    static constexpr uint32_t SMEM_BYTES = RED_OFF + (NSB - 1) * BM * 8;
    static constexpr uint32_t SMEM_ALLOC = SMEM_BYTES + 1024;
    static_assert(SMEM_ALLOC <= 227u * 1024u, "shared memory budget");
};
}  // namespace w

template <int KF, int NW, int EMU>
__global__ void __launch_bounds__(w::NTHREADS, 1)
tcw_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
           const __grid_constant__ CUtensorMap tmq_n, const __grid_constant__ CUtensorMap tmk_n,
           const float* __restrict__ u, int64_t nq, uint32_t idesc, Sched sc, RowEpilogue ep,
           double* __restrict__ part, int* __restrict__ status) {
    using C = w::Cfg<KF, NW>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sQ = base;
    uint8_t* sR = base + C::RING_OFF;
    float* sU = (float*)(base + C::U_OFF);
    uint64_t* bars = (uint64_t*)(base + C::BAR_OFF);
    uint64_t* kfull = bars;
    uint64_t* kempty = kfull + C::SLOTS;
    uint64_t* ufull = kempty + C::SLOTS;
    uint64_t* uempty = ufull + URING;
    uint64_t* qfull = uempty + URING;
    uint64_t* qempty = qfull + 1;
    uint64_t* sfull = qempty + 1;
    uint64_t* sempty = sfull + w::NSB;
    uint64_t* rfull = sempty + w::NSB;
    uint64_t* rempty = rfull + 1;
    uint64_t* done = rempty + 1;
    uint32_t* tmem_slot = (uint32_t*)(base + C::MISC_OFF);
    volatile int* abort = (volatile int*)(base + C::MISC_OFF + 4);
    double* red = (double*)(base + C::RED_OFF);   // [NSB - 1][BM]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int cta = blockIdx.x;

    if (threadIdx.x == 0) {
        for (int i = 0; i < C::SLOTS; ++i) {
            ptx::mbar_init(&kfull[i], 1);
            ptx::mbar_init(&kempty[i], 1);
        }
        for (int i = 0; i < URING; ++i) {
            ptx::mbar_init(&ufull[i], 1);
            ptx::mbar_init(&uempty[i], 4);      // the 4 warps of the warpgroup of tile m = i (mod 4)
        }
        ptx::mbar_init(qfull, 1);
        ptx::mbar_init(qempty, 2);                  // both issuers, at every row-tile end
        for (int i = 0; i < w::NSB; ++i) {
            ptx::mbar_init(&sfull[i], 1);
            ptx::mbar_init(&sempty[i], 4);
        }
        ptx::mbar_init(rfull, (w::NSB - 1) * w::BM);   // every thread of warpgroups 1-3
        ptx::mbar_init(rempty, w::BM);                 // every thread of warpgroup 0
        ptx::mbar_init(&done[0], 1);
        ptx::mbar_init(&done[1], 1);
        *abort = 0;
        ptx::fence_mbar_init();
    }
    if (warp == w::MMA_WARP) {
        ptx::tmem_alloc(tmem_slot, TMEM_COLS);
        ptx::tmem_relinquish();
    }
    if (warp == w::TMA_WARP && lane == 0) {
        ptx::prefetch_tmap(&tmq);
        ptx::prefetch_tmap(&tmk);
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == w::TMA_WARP || warp == w::TMA_WARP_ODD) {
        if (lane == 0) {
            const int pp = warp == w::TMA_WARP ? 0 : 1;   // this producer's tile parity
            bool pacing = true;                            // (the even-tile producer paces)
            int64_t paced = -1;
            uint32_t qcount = 0;
            int64_t cur_rt = -1;
            for (Walk wk(sc, cta); !wk.done(); wk.next()) {
                const int64_t m = wk.s, rt = wk.rt, jt = wk.jt;
                if (pp == 0 && rt != cur_rt) {
                    if (qcount > 0 && !ptx::wait_bounded(qempty, (qcount - 1) & 1, abort, status, WAIT_LIMIT_NS)) break;
                    ptx::mbar_expect_tx(qfull, C::Q_BYTES);
                    for (int kb = 0; kb < KF; ++kb)
                        ptx::tma_load_2d(sQ + kb * w::BM * 128, &tmq, qfull, kb * 64, (int)(rt * w::BM));
                    if (NW) ptx::tma_load_2d(sQ + KF * w::BM * 128, &tmq_n, qfull, KF * 64, (int)(rt * w::BM));
                    cur_rt = rt;
                    ++qcount;
                }
                if ((int)(m & 1) != pp) continue;
                if (pp == 0 && pacing) pacing = pace(sc, m, jt, abort, paced);
                bool ok = true;
                for (int kb = 0; kb < C::NB; ++kb) {
                    // position in this pipeline's sub-ring, consumed in order by one issuer
                    const int64_t pos = (m >> 1) * C::NB + kb;
                    const int slot = pp * C::SH + (int)(pos % C::SH);
                    const uint32_t kph = (uint32_t)((pos / C::SH) & 1);
                    if (!ptx::wait_bounded(&kempty[slot], kph ^ 1, abort, status, WAIT_LIMIT_NS)) { ok = false; break; }
                    uint8_t* dst = sR + slot * w::SLOT_BYTES;
                    if (kb < KF) {
                        ptx::mbar_expect_tx(&kfull[slot], w::SLOT_BYTES);
                        ptx::tma_load_2d(dst, &tmk, &kfull[slot], kb * 64, (int)(jt * w::BN));
                    } else {
                        ptx::mbar_expect_tx(&kfull[slot], C::NARROW_BYTES);
                        ptx::tma_load_2d(dst, &tmk_n, &kfull[slot], KF * 64, (int)(jt * w::BN));
                    }
                }
                if (!ok) break;
                const int us = (int)(m & (URING - 1));
                const uint32_t uph = (uint32_t)((m / URING) & 1);
                if (!ptx::wait_bounded(&uempty[us], uph ^ 1, abort, status, WAIT_LIMIT_NS)) break;
                ptx::mbar_expect_tx(&ufull[us], U_BYTES);
                ptx::bulk_load(sU + us * w::BN, u + jt * w::BN, U_BYTES, &ufull[us]);
            }
        }
    } else if (warp == w::MMA_WARP || warp == w::MMA_WARP + 1) {
        if (lane == 0) {
            const int pp = warp - w::MMA_WARP;             // this issuer's tile parity
            const uint32_t q_base = ptx::smem_u32(sQ), r_base = ptx::smem_u32(sR);
            uint32_t qcount = 0;
            int64_t cur_rt = -1;
            for (Walk wk(sc, cta); !wk.done(); wk.next()) {
                const int64_t m = wk.s, rt = wk.rt;
                const int b = (int)(m % w::NSB);
                if (rt != cur_rt) {
                    if (!ptx::wait_bounded(qfull, qcount & 1, abort, status, WAIT_LIMIT_NS)) break;
                    ++qcount;
                    cur_rt = rt;
                }
                if ((int)(m & 1) == pp) {
                    if (!ptx::wait_bounded(&sempty[b], (uint32_t)(((m / w::NSB) & 1) ^ 1), abort, status, WAIT_LIMIT_NS)) break;
                    bool ok = true;
                    for (int kb = 0; kb < C::NB; ++kb) {
                        const int64_t pos = (m >> 1) * C::NB + kb;
                        const int slot = pp * C::SH + (int)(pos % C::SH);
                        const uint32_t kph = (uint32_t)((pos / C::SH) & 1);
                        if (!ptx::wait_bounded(&kfull[slot], kph, abort, status, WAIT_LIMIT_NS)) { ok = false; break; }
                        ptx::tc_fence_after();
                        const uint32_t ka = r_base + slot * w::SLOT_BYTES;
                        if (kb < KF) {
                            const uint32_t qa = q_base + kb * w::BM * 128;
#pragma unroll
                            for (int ks = 0; ks < 4; ++ks)
                                ptx::umma_ss(tmem + b * w::BN, ptx::sw128_kmajor_desc(qa + ks * 32),
                                             ptx::sw128_kmajor_desc(ka + ks * 32), idesc, (kb | ks) ? 1u : 0u);
                        } else {
                            const uint32_t qa = q_base + KF * w::BM * 128;
#pragma unroll
                            for (int ks = 0; ks < NW / 16; ++ks) {
                                const uint64_t dq = NW == 32 ? ptx::sw64_kmajor_desc(qa + ks * 32) : ptx::sw32_kmajor_desc(qa + ks * 32);
                                const uint64_t dk = NW == 32 ? ptx::sw64_kmajor_desc(ka + ks * 32) : ptx::sw32_kmajor_desc(ka + ks * 32);
                                ptx::umma_ss(tmem + b * w::BN, dq, dk, idesc, 1u);
                            }
                        }
                        ptx::umma_commit(&kempty[slot]);
                    }
                    if (!ok) break;
                    ptx::umma_commit(&sfull[b]);
                }
                if (wk.seg_last()) ptx::umma_commit(qempty);
            }
            ptx::umma_commit(&done[pp]);
            ptx::wait_bounded(&done[pp], 0, abort, status, WAIT_LIMIT_NS);
        }
    } else if (warp < 16) {
        // ---- epilogue: warpgroup wg owns S buffer wg and the tiles m = wg (mod 4)
        const int wg = warp >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
        double acc = 0.0;
        uint32_t segs = 0;
        bool alive = true;
        for (Walk wk(sc, cta); !wk.done() && alive; wk.next()) {
            const int64_t m = wk.s, rt = wk.rt;
            if ((int)(m % w::NSB) == wg) {
                const uint32_t use = (uint32_t)(m / w::NSB);
                const int us = (int)(m & (URING - 1));
                if (!ptx::wait_bounded(&ufull[us], (uint32_t)((m / URING) & 1), abort, status, WAIT_LIMIT_NS)) { alive = false; break; }
                if (!ptx::wait_bounded(&sfull[wg], use & 1, abort, status, WAIT_LIMIT_NS)) { alive = false; break; }
                ptx::tc_fence_after();
                const float* ut = sU + us * w::BN;
                uint64_t acc_a = 0, acc_b = 0;
                uint32_t va[16], vb[16];
                const uint32_t tb = t_lane + wg * w::BN;
                ptx::tmem_ld16(tb, va);
                ptx::tmem_wait_ld16(va);
#pragma unroll 1
                for (int c = 0; c < w::BN / 16; c += 2) {
                    ptx::tmem_ld16(tb + (c + 1) * 16, vb);
                    chunk16_r1<EMU>(va, ut + c * 16, acc_a, acc_b);
                    ptx::tmem_wait_ld16(vb);
                    if (c + 2 < w::BN / 16) ptx::tmem_ld16(tb + (c + 2) * 16, va);
                    chunk16_r1<EMU>(vb, ut + (c + 1) * 16, acc_a, acc_b);
                    if (c + 2 < w::BN / 16) ptx::tmem_wait_ld16(va);
                }
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    ptx::mbar_arrive(&sempty[wg]);
                    ptx::mbar_arrive(&uempty[us]);
                }
                uint32_t a0, a1, b0, b1;
                ptx::unpack2(acc_a, a0, a1);
                ptx::unpack2(acc_b, b0, b1);
                acc += (double)((__uint_as_float(a0) + __uint_as_float(a1)) + (__uint_as_float(b0) + __uint_as_float(b1)));
            }
            if (wk.seg_last()) {
                // the four warpgroups' partial row sums meet in warpgroup 0
                const uint32_t ph = segs & 1;
                if (wg > 0) {
                    if (!ptx::wait_bounded(rempty, ph ^ 1, abort, status, WAIT_LIMIT_NS)) { alive = false; break; }
                    red[(wg - 1) * w::BM + row] = acc;
                    ptx::mbar_arrive(rfull);
                } else {
                    if (!ptx::wait_bounded(rfull, ph, abort, status, WAIT_LIMIT_NS)) { alive = false; break; }
                    const double tot = acc + red[row] + red[w::BM + row] + red[2 * w::BM + row];
                    ptx::mbar_arrive(rempty);
                    const int64_t gi = rt * w::BM + row;
                    if (gi < nq) {
                        if (wk.seg_full()) store_out(ep, gi, 0, tot);
                        else part[((int64_t)cta * 2 + wk.slot()) * w::BM + row] = tot;
                    }
                }
                acc = 0.0;
                ++segs;
            }
        }
        ptx::tc_fence_before();
    }
    __syncthreads();
    if (warp == w::MMA_WARP) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// Fix-up of the wide kernel: 128-row tiles.
__global__ void tcw_fixup_kernel(const double* __restrict__ part, Sched sc, int64_t nq, RowEpilogue ep) {
    const int64_t rt = blockIdx.x;
    for (int r = threadIdx.x; r < w::BM; r += blockDim.x) {
        const int64_t gi = rt * w::BM + r;
        if (gi >= nq) continue;
        double sum = 0.0;
        const bool cut = for_each_cut_owner(sc, rt, [&](int c, int slot) {
            sum += part[((int64_t)c * 2 + slot) * w::BM + r];
        });
        if (cut) store_out(ep, gi, 0, sum);
    }
}

}  // namespace tc

// ---- host side -----------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static int get_encode(EncodeTiledFn* fn) {
    static EncodeTiledFn cached = nullptr;
    if (!cached) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        FD_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !p)
            return set_error(FD_ERR_CUDA, "cuTensorMapEncodeTiled entry point not found");
        cached = (EncodeTiledFn)p;
    }
    *fn = cached;
    return FD_OK;
}

int make_tile_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int box_rows, bool f16,
                  int box_cols) {
    EncodeTiledFn enc;
    FD_TRY(get_encode(&enc));
    FD_CHECK_ARG(((uintptr_t)ptr & 15) == 0, "tile operand must be 16-byte aligned");
    FD_CHECK_ARG((cols * 2) % 16 == 0, "tile operand row pitch must be a multiple of 16 bytes");
    FD_CHECK_ARG(box_cols == 64 || box_cols == 32 || box_cols == 16, "box width %d", box_cols);
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapSwizzle sw = box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : (box_cols == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
    CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                     const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(FD_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return FD_OK;
}

void split_kd(int kd, int* kf, int* nw) {
    *kf = kd / 64;
    *nw = kd % 64;
    if (*nw == 48) { *kf += 1; *nw = 0; }
}

int num_sms() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

// cross-CTA partials, then one 256-byte line for the lockstep pacing counter
size_t tc_workspace_bytes(int64_t nq, int64_t nk, int rc) {
    (void)nq; (void)nk; (void)rc;
    return align256(sizeof(double) * 2 * (size_t)num_sms() * tc::ROWS) + 256;
}

// Key tiles per pacing chunk: about 8 MB of key-side bytes.
int64_t pace_tiles(size_t bytes_per_key_tile) {
    const int64_t t = (int64_t)((8u << 20) / (bytes_per_key_tile ? bytes_per_key_tile : 1));
    return t < 8 ? 8 : t;
}

struct TcArgs {
    CUtensorMap mq, mk, mqn, mkn;
    const float* u;
    int64_t nq;
    uint32_t idesc;
    tc::Sched sc;
    RowEpilogue ep;
    double* part;
};

template <int KF, int NW, int EMU>
static int launch_tc_kb(const TcArgs& a, cudaStream_t s) {
    using C = tc::Cfg<KF, NW>;
    FD_CUDA_TRY(cudaFuncSetAttribute(tc::tc_kernel<KF, NW, EMU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)C::SMEM_ALLOC));
    int* status = nullptr;
    FD_TRY(status_word(&status));
    tc::tc_kernel<KF, NW, EMU><<<a.sc.grid, tc::NTHREADS, C::SMEM_ALLOC, s>>>(a.mq, a.mk, a.mqn, a.mkn, a.u, a.nq,
                                                                              a.idesc, a.sc, a.ep, a.part, status);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

// Columns per 16 whose exp2 runs on the FMA pipe instead of MUFU (degree-4
// polynomial, relative error 3.6e-6): 4 by default for the 16-bit tiles, where
// MUFU is the limit; 0 for the fp32-class tiles (their error budget is 1e-5).
// fd_set_exp2_fma_cols overrides the 16-bit default (0, 2, 4, 6 or 8).
static int g_exp2_fma_cols = -1;

static int exp2_fma_cols(int tile) {
    if (tile == FD_TILE_F16X3) return 0;
    return g_exp2_fma_cols >= 0 ? g_exp2_fma_cols : 4;
}

template <int KF, int NW>
static int launch_tc_emu(const TcArgs& a, int emu, cudaStream_t s) {
    switch (emu) {
        case 2: return launch_tc_kb<KF, NW, 2>(a, s);
        case 4: return launch_tc_kb<KF, NW, 4>(a, s);
        case 6: return launch_tc_kb<KF, NW, 6>(a, s);
        case 8: return launch_tc_kb<KF, NW, 8>(a, s);
        default: return launch_tc_kb<KF, NW, 0>(a, s);
    }
}

template <int KF, int NW, int EMU>
static int launch_tcw_kb(const TcArgs& a, cudaStream_t s) {
    using C = tc::w::Cfg<KF, NW>;
    FD_CUDA_TRY(cudaFuncSetAttribute(tc::tcw_kernel<KF, NW, EMU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)C::SMEM_ALLOC));
    int* status = nullptr;
    FD_TRY(status_word(&status));
    tc::tcw_kernel<KF, NW, EMU><<<a.sc.grid, tc::w::NTHREADS, C::SMEM_ALLOC, s>>>(
        a.mq, a.mk, a.mqn, a.mkn, a.u, a.nq, a.idesc, a.sc, a.ep, a.part, status);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

template <int KF, int NW>
static int launch_tcw_emu(const TcArgs& a, int emu, cudaStream_t s) {
    return emu ? launch_tcw_kb<KF, NW, 4>(a, s) : launch_tcw_kb<KF, NW, 0>(a, s);
}

// Operand rows of 224..416 columns (fp32-class tiles of d = 68..136; 16-bit
// tiles of d = 203..410): 128-row query tiles, key tiles streamed by box.
static int launch_tc_wide(const void* qop, int64_t nq, const void* kop, int64_t nk, int kd, int tile,
                          const void* rhs, const RowEpilogue& ep, void* ws, size_t ws_bytes, cudaStream_t s) {
    int kf = 0, nw = 0;
    split_kd(kd, &kf, &nw);
    const size_t need = tc_workspace_bytes(nq, nk, 1);
    if (ws_bytes < need) return set_error(FD_ERR_WORKSPACE, "16-bit tile path: workspace %zu B < %zu B", ws_bytes, need);
    TcArgs a;
    const bool f16 = tile != FD_TILE_BF16;
    FD_TRY(make_tile_map(&a.mq, qop, nq, kd, tc::w::BM, f16));
    FD_TRY(make_tile_map(&a.mk, kop, nk, kd, tc::w::BN, f16));
    a.mqn = a.mq;
    a.mkn = a.mk;
    if (nw) {
        FD_TRY(make_tile_map(&a.mqn, qop, nq, kd, tc::w::BM, f16, nw));
        FD_TRY(make_tile_map(&a.mkn, kop, nk, kd, tc::w::BN, f16, nw));
    }
    a.idesc = ptx::idesc_f32acc(tc::w::BM, tc::w::BN, f16);
    a.sc = tc::Sched::make(cdiv(nq, tc::w::BM), cdiv(nk, tc::w::BN), num_sms(), (size_t)nk * kd * 2);
    a.part = (double*)ws;
    if (a.sc.full > 0) {
        a.sc.sync = (unsigned*)((uint8_t*)ws + need - 256);
        a.sc.pace_tiles = pace_tiles((size_t)tc::w::BN * kd * 2 + tc::w::BN * 4);
        FD_CUDA_TRY(cudaMemsetAsync(a.sc.sync, 0, sizeof(unsigned), s));
    }
    a.u = (const float*)rhs;
    a.nq = nq;
    a.ep = ep;
    const int emu = exp2_fma_cols(tile) ? 1 : 0;
    switch (kf * 100 + nw) {
        case 332: FD_TRY((launch_tcw_emu<3, 32>(a, emu, s))); break;
        case 400: FD_TRY((launch_tcw_emu<4, 0>(a, emu, s))); break;
        case 416: FD_TRY((launch_tcw_emu<4, 16>(a, emu, s))); break;
        case 432: FD_TRY((launch_tcw_emu<4, 32>(a, emu, s))); break;
        case 500: FD_TRY((launch_tcw_emu<5, 0>(a, emu, s))); break;
        case 516: FD_TRY((launch_tcw_emu<5, 16>(a, emu, s))); break;
        case 532: FD_TRY((launch_tcw_emu<5, 32>(a, emu, s))); break;
        case 600: FD_TRY((launch_tcw_emu<6, 0>(a, emu, s))); break;
        case 616: FD_TRY((launch_tcw_emu<6, 16>(a, emu, s))); break;
        case 632: FD_TRY((launch_tcw_emu<6, 32>(a, emu, s))); break;
        default: return set_error(FD_ERR_UNSUPPORTED, "tensor-core tile path: no kernel for kd=%d", kd);
    }
    tc::tcw_fixup_kernel<<<(unsigned)cdiv(nq, tc::w::BM), 256, 0, s>>>(a.part, a.sc, nq, ep);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

int launch_tc(const void* qop, int64_t nq, const void* kop, int64_t nk, int d, int tile,
              const void* rhs, int rc, const RowEpilogue& ep, void* ws, size_t ws_bytes, cudaStream_t s) {
    if (nq == 0) return FD_OK;
    if (nk == 0) return launch_zero_rows(nq, rc, ep, s);
    if (rc != 1) return set_error(FD_ERR_UNSUPPORTED, "16-bit tile path: block right-hand sides not built yet");
    const int kd = kd_tile(tile, d);
    int kf = 0, nw = 0;
    split_kd(kd, &kf, &nw);
    if (kd > 416) return set_error(FD_ERR_UNSUPPORTED, "tensor-core tile path: operand rows of %d columns (max 416)", kd);
    if (kd > 208) return launch_tc_wide(qop, nq, kop, nk, kd, tile, rhs, ep, ws, ws_bytes, s);
    const size_t need = tc_workspace_bytes(nq, nk, rc);
    if (ws_bytes < need) return set_error(FD_ERR_WORKSPACE, "16-bit tile path: workspace %zu B < %zu B", ws_bytes, need);
    TcArgs a;
    const bool f16 = tile != FD_TILE_BF16;
    FD_TRY(make_tile_map(&a.mq, qop, nq, kd, tc::BM, f16));
    FD_TRY(make_tile_map(&a.mk, kop, nk, kd, tc::BN, f16));
    a.mqn = a.mq;
    a.mkn = a.mk;
    if (nw) {
        FD_TRY(make_tile_map(&a.mqn, qop, nq, kd, tc::BM, f16, nw));
        FD_TRY(make_tile_map(&a.mkn, kop, nk, kd, tc::BN, f16, nw));
    }
    a.idesc = ptx::idesc_f32acc(tc::BM, tc::BN, f16);
    a.sc = tc::Sched::make(cdiv(nq, tc::ROWS), cdiv(nk, tc::BN), num_sms(), (size_t)nk * kd * 2);
    a.part = (double*)ws;
    if (a.sc.full > 0) {
        a.sc.sync = (unsigned*)((uint8_t*)ws + need - 256);
        a.sc.pace_tiles = pace_tiles((size_t)tc::BN * kd * 2 + tc::BN * 4);
        FD_CUDA_TRY(cudaMemsetAsync(a.sc.sync, 0, sizeof(unsigned), s));
    }
    a.u = (const float*)rhs;
    a.nq = nq;
    a.ep = ep;
    const int emu = exp2_fma_cols(tile);
    switch (kf * 100 + nw) {
        case 16: FD_TRY((launch_tc_emu<0, 16>(a, emu, s))); break;
        case 32: FD_TRY((launch_tc_emu<0, 32>(a, emu, s))); break;
        case 100: FD_TRY((launch_tc_emu<1, 0>(a, emu, s))); break;
        case 116: FD_TRY((launch_tc_emu<1, 16>(a, emu, s))); break;
        case 132: FD_TRY((launch_tc_emu<1, 32>(a, emu, s))); break;
        case 200: FD_TRY((launch_tc_emu<2, 0>(a, emu, s))); break;
        case 216: FD_TRY((launch_tc_emu<2, 16>(a, emu, s))); break;
        case 232: FD_TRY((launch_tc_emu<2, 32>(a, emu, s))); break;
        case 300: FD_TRY((launch_tc_emu<3, 0>(a, emu, s))); break;
        case 316: FD_TRY((launch_tc_emu<3, 16>(a, emu, s))); break;
        default: return set_error(FD_ERR_UNSUPPORTED, "tensor-core tile path: no kernel for kd=%d", kd);
    }
    tc::tc_fixup_kernel<<<(unsigned)cdiv(nq, tc::ROWS), 256, 0, s>>>(a.part, a.sc, nq, ep);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

int status_word(int** ptr) {
    static int* cached[64] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    FD_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(FD_ERR_ARG, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!cached[dev]) {
        int* p = nullptr;
        FD_CUDA_TRY(cudaGetSymbolAddress((void**)&p, g_fd_status));
        cached[dev] = p;
    }
    *ptr = cached[dev];
    return FD_OK;
}

int read_and_clear_status(cudaStream_t s, int* status) {
    int zero = 0;
    FD_CUDA_TRY(cudaMemcpyFromSymbolAsync(status, g_fd_status, sizeof(int), 0, cudaMemcpyDeviceToHost, s));
    FD_CUDA_TRY(cudaMemcpyToSymbolAsync(g_fd_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s));
    FD_CUDA_TRY(cudaStreamSynchronize(s));
    return FD_OK;
}

}  // namespace fd

namespace {
// One bounded wait on an mbarrier that nothing arrives at: the failure path of
// every pipeline wait in the kernels (limit, abort flag, status word), without
// a fault.
__global__ void wait_selftest_kernel(int* status, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        fd::ptx::mbar_init(&bar, 1);
        abort_flag = 0;
        fd::ptx::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) fd::ptx::wait_bounded(&bar, 0, &abort_flag, status, limit_ns);
}
}  // namespace

extern "C" int fd_selftest_wait_timeout(int64_t limit_ns, void* stream) {
    FD_CHECK_ARG(limit_ns >= 1000000 && limit_ns <= 2000000000, "fd_selftest_wait_timeout: limit %lld ns "
                 "(1e6..2e9)", (long long)limit_ns);
    int* status = nullptr;
    FD_TRY(fd::status_word(&status));
    wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(status, (uint64_t)limit_ns);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

extern "C" int fd_set_exp2_fma_cols(int cols) {
    FD_CHECK_ARG(cols == -1 || cols == 0 || cols == 2 || cols == 4 || cols == 6 || cols == 8,
                 "fd_set_exp2_fma_cols: %d (-1 = default, or 0, 2, 4, 6, 8)", cols);
    fd::g_exp2_fma_cols = cols;
    return FD_OK;
}

namespace {
__global__ void exp2_poly_selftest_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ y) {
    for (int64_t i = 2 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x); i < n;
         i += 2 * (int64_t)gridDim.x * blockDim.x) {
        const float a = x[i], b = i + 1 < n ? x[i + 1] : 0.0f;
        uint32_t lo, hi;
        fd::ptx::unpack2(fd::tc::exp2_poly2(__float_as_uint(a), __float_as_uint(b)), lo, hi);
        y[i] = __uint_as_float(lo);
        if (i + 1 < n) y[i + 1] = __uint_as_float(hi);
    }
}
}  // namespace

extern "C" int fd_selftest_exp2_poly(const float* x, int64_t n, float* y, void* stream) {
    FD_CHECK_ARG(n >= 0 && (n == 0 || (x && y)), "fd_selftest_exp2_poly: bad arguments");
    if (n == 0) return FD_OK;
    const int64_t pairs = (n + 1) / 2;
    const int grid = (int)((pairs + 255) / 256 < 148 * 8 ? (pairs + 255) / 256 : 148 * 8);
    exp2_poly_selftest_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, n, y);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}
