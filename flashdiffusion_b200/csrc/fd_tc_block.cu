// Block right-hand sides (r > 1) on the 16-bit tensor-core path: two tcgen05
// GEMMs per key tile.
//
//   S = Q~ K~^T            (tcgen05.mma, A and B from shared memory, fp32 in TMEM)
//   P = 2^S                (epilogue warps: MUFU ex2, split P = P_hi + P_lo into two
//                           fp16 parts written back to TMEM over S columns each
//                           warpgroup has already read)
//   O += P_hi U_hi + P_hi U_lo + P_lo U_hi
//                          (two tcgen05.mma per 16 keys, A from TMEM: P_hi times
//                           the stacked [U_hi; U_lo] tile (N = 2r) into two
//                           accumulator halves, then P_lo U_hi; the halves are
//                           summed when O is read): fp32-class products from
//                           fp16 operands, so the block path keeps the accuracy
//                           of the r = 1 path (which multiplies in fp32)
//
// U = diag(col_scale * col_h) V, stored transposed as fp16 hi/lo pairs with one
// power-of-two scale per column (so every column uses the fp16 range; the
// scale is undone in the output epilogue).  There is no online softmax: the row scale is a
// known vector, applied once per output row.
//
// CTA = 128 query rows x stream of 128-key tiles.  Warp roles (18 warps):
//   warps 0-11  three epilogue warpgroups; warpgroup w exponentiates the key
//               tiles m = w (mod 3) in its own TMEM S/P buffer (3 x 128 columns,
//               plus 3 x 32 accumulator columns: 480 of the 512 TMEM columns)
//   warp  12    TMA producer: query tile per row tile; per key tile the K
//               box(es) into the K ring and the 64-key boxes of U_hi^T and
//               U_lo^T into the U ring (no multicast)
//   warps 13-14 Q.K^T issuers (even / odd tiles)
//   warps 15-16 P.U issuers, one per accumulator chain: each tcgen05.mma
//               costs its issuing thread about 100 cycles whatever its size,
//               so independent chains get their own issuing warps
// The persistent work split and the deterministic cross-CTA fix-up are the
// ones of the r = 1 kernel (fd_tc.cu).
#include "fd_tc_common.cuh"

namespace fd {
namespace tcb {

// Optional wait-time accounting (build with -DFD_PROFILE_WAITS): cycles that
// lane 0 of each warp of CTA 0 spends in each pipeline wait, by wait site.
#ifdef FD_PROFILE_WAITS
__device__ unsigned long long g_wait_cycles[16];
__device__ __forceinline__ bool timed_wait(int slot, uint64_t* b, uint32_t ph, volatile int* a, int* st,
                                           uint64_t lim) {
    const long long t0 = clock64();
    const bool ok = ptx::wait_bounded(b, ph, a, st, lim);
    if (blockIdx.x == 0 && (threadIdx.x & 31) == 0)
        atomicAdd(&g_wait_cycles[slot], (unsigned long long)(clock64() - t0));
    return ok;
}
#define FD_WAIT(slot, ...) timed_wait(slot, __VA_ARGS__)
#define FD_SPAN_BEGIN const long long span_t0 = clock64()
#define FD_SPAN_END(slot) \
    if (blockIdx.x == 0) atomicAdd(&g_wait_cycles[slot], (unsigned long long)(clock64() - span_t0))
#else
#define FD_WAIT(slot, ...) ptx::wait_bounded(__VA_ARGS__)
#define FD_SPAN_BEGIN
#define FD_SPAN_END(slot)
#endif

using tc::Sched;
using tc::Walk;
using tc::for_each_cut_owner;

constexpr int BM = 128;
constexpr int BN = 128;                    // keys per tile (N of Q.K^T, K of P.U)
constexpr int NEPI_WG = 3;                 // epilogue warpgroups = TMEM S/P buffers
constexpr int TMA_WARP = 12;
constexpr int MMA_WARP = 13;               // Q.K^T issuer of even tiles (and TMEM owner); 14: odd tiles
constexpr int PV_WARP0 = 15;               // P_hi . [U_hi; U_lo] issuer
constexpr int PV_WARP1 = 16;               // P_lo . U_hi issuer
constexpr int UTMA_WARP = 17;              // U^T tile loads (own thread, so a full U ring never delays K)
constexpr int NTHREADS = 18 * 32;
constexpr uint32_t BOX_BYTES = 128 * 128;  // query box: 128 rows x 64 16-bit columns
constexpr uint32_t KBOX_BYTES = BN * 128;  // key box: BN rows x 64 16-bit columns
constexpr uint32_t TMEM_COLS = 512;
constexpr int NSB = NEPI_WG;               // TMEM S/P buffers of BN columns, one per epilogue warpgroup
constexpr uint32_t O_COL = NSB * BN;       // accumulators O1 [384, 384 + 2 RP) and O2 [384 + 2 RP, 384 + 4 RP)
// O is restarted every `ogroup` key tiles and the group sums are added on the
// CUDA cores in fp32 (round to nearest): the tensor-core accumulation rounds
// toward zero, so one TMEM accumulator summed over thousands of P.U products
// drifts low (measured: a relative bias of 1.7e-3 after 2,048 key tiles,
// linear in the number of accumulation steps).  With groups of g tiles the
// bias is about 7.5e-7 g, independent of the number of keys.
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;

template <int KF, int NW, int RP>
struct Cfg {
    using G = tc::Geo<KF, NW>;
    static constexpr uint32_t Q_BYTES = G::bytes(BM);
    static constexpr uint32_t UT_BOX = RP * 128;                 // RP rows x 64 keys
    // two rings: K tiles (released as soon as Q.K^T is done) and U^T tiles
    // (U_hi^T and U_lo^T, 2 boxes each; released after P.U, i.e. after the epilogue)
    // Wide operands (fp32-class tiles of d = 68..136: rows of 224..416 columns):
    // a whole key tile per ring stage would leave no room for a second stage,
    // so the K ring holds single 64-column boxes (the narrow box in a slot of
    // its own) and one issuer consumes them in order.
    static constexpr bool WIDE = KF * 64 + NW > 208;
    static constexpr uint32_t STAGE_BYTES = WIDE ? KBOX_BYTES : G::bytes(BN);
    static constexpr uint32_t USTAGE_BYTES = 4 * UT_BOX;
    static constexpr uint32_t BUDGET = 222u * 1024u - Q_BYTES;
    static constexpr uint32_t ACC_BYTES = RP * BM * 4;     // running O sums of the segment
    // U^T tiles live from their load to their P.U: 4 stages unless that leaves
    // fewer than 3 K stages (2 for the wide operands)
    static constexpr int USTAGES =
        WIDE ? 2 : ((BUDGET - ACC_BYTES - 4 * USTAGE_BYTES) / STAGE_BYTES >= 3 ? 4 : 3);
    static constexpr int K_RAW = (int)((BUDGET - ACC_BYTES - USTAGES * USTAGE_BYTES) / STAGE_BYTES);
    static constexpr int STAGES = K_RAW > (WIDE ? 8 : 6) ? (WIDE ? 8 : 6) : (K_RAW < 2 ? 2 : K_RAW);
    static_assert(!WIDE || STAGES >= 3, "wide operands need at least 3 box slots");
    static constexpr uint32_t U_OFF = Q_BYTES + STAGES * STAGE_BYTES;
    static constexpr uint32_t ACC_OFF = U_OFF + USTAGES * USTAGE_BYTES;
    static constexpr uint32_t BAR_OFF = ACC_OFF + ACC_BYTES;
    // kfull[S], kempty[S], ufull[U], uempty[U], qfull, qempty, sfull[3], sempty[3], pfull[3], ofull[3],
    // oempty, done[4]
    static constexpr int NBARS = 2 * STAGES + 2 * USTAGES + 2 + 4 * NSB + 5;
    static constexpr uint32_t SEQ_OFF = BAR_OFF + NBARS * 8;
    static constexpr uint32_t MISC_OFF = SEQ_OFF + BM * 4;
    static constexpr uint32_t SMEM_BYTES = MISC_OFF + 16;
    static constexpr uint32_t SMEM_ALLOC = SMEM_BYTES + 1024;
    static_assert(SMEM_ALLOC <= 227 * 1024, "shared memory budget");
    static_assert(O_COL + 4 * RP <= TMEM_COLS, "TMEM budget");
};

// Load `RP / 4` consecutive O columns of this thread's row.
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&o)[N]);
template <>
__device__ __forceinline__ void tmem_ld_cols<16>(uint32_t taddr, float (&o)[16]) {
    uint32_t v[16];
    ptx::tmem_ld16(taddr, v);
    ptx::tmem_wait_ld16(v);
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = __uint_as_float(v[i]);
}
template <>
__device__ __forceinline__ void tmem_ld_cols<8>(uint32_t taddr, float (&o)[8]) {
    uint32_t v[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7])
                 :: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = __uint_as_float(v[i]);
}
template <>
__device__ __forceinline__ void tmem_ld_cols<4>(uint32_t taddr, float (&o)[4]) {
    uint32_t v[4];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]) : "r"(taddr) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]) :: "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = __uint_as_float(v[i]);
}

// 32 lanes x 8 columns <- 8 registers (16 fp16 values of P per thread).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

// 16 S values -> P = 2^S as fp16 hi and lo parts (P - hi, exact in fp32 before
// rounding), each packed in 8 registers with key 2c in the low half.
__device__ __forceinline__ void exp2_to_f16x2(const uint32_t (&v)[16], uint32_t (&hi)[8], uint32_t (&lo)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float e0 = ptx::ex2_mufu(__uint_as_float(v[2 * i]));
        const float e1 = ptx::ex2_mufu(__uint_as_float(v[2 * i + 1]));
        const __half2 h = __floats2half2_rn(e0, e1);
        const float2 hf = __half22float2(h);
        const __half2 l = __floats2half2_rn(e0 - hf.x, e1 - hf.y);
        hi[i] = *reinterpret_cast<const uint32_t*>(&h);
        lo[i] = *reinterpret_cast<const uint32_t*>(&l);
    }
}

// 16 S values -> P = 2^S rounded once to fp16, 8 registers, key 2c in the low half.
__device__ __forceinline__ void exp2_to_f16(const uint32_t (&v)[16], uint32_t (&p)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const __half2 h = __floats2half2_rn(ptx::ex2_mufu(__uint_as_float(v[2 * i])),
                                            ptx::ex2_mufu(__uint_as_float(v[2 * i + 1])));
        p[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
}

template <int KF, int NW, int RP>
__global__ void __launch_bounds__(NTHREADS, 1)
tc_block_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                const __grid_constant__ CUtensorMap tmq_n, const __grid_constant__ CUtensorMap tmk_n,
                const __grid_constant__ CUtensorMap tmu, const float* __restrict__ colscale, int rc,
                int64_t nq, uint32_t idesc_qk, uint32_t idesc_pv, Sched sc, RowEpilogue ep,
                double* __restrict__ part, int* __restrict__ status, uint32_t idesc_pv2, int ogroup, int three) {
    using C = Cfg<KF, NW, RP>;
    using G = typename C::G;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sQ = base;
    uint8_t* sK = base + C::Q_BYTES;
    uint64_t* bars = (uint64_t*)(base + C::BAR_OFF);
    uint64_t* kfull = bars;
    uint64_t* kempty = kfull + C::STAGES;
    uint64_t* ufull = kempty + C::STAGES;
    uint64_t* uempty = ufull + C::USTAGES;
    uint64_t* qfull = uempty + C::USTAGES;
    uint64_t* qempty = qfull + 1;
    uint64_t* sfull = qfull + 2;
    uint64_t* sempty = sfull + NSB;
    uint64_t* pfull = sempty + NSB;
    uint64_t* ofull = pfull + NSB;          // one per epilogue warpgroup: the group's reader
    uint64_t* oempty = ofull + NSB;
    uint64_t* done = oempty + 1;
    uint32_t* aseq = (uint32_t*)(base + C::SEQ_OFF);   // per row: O groups added into sacc
    uint32_t* tmem_slot = (uint32_t*)(base + C::MISC_OFF);
    volatile int* abort = (volatile int*)(base + C::MISC_OFF + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
#ifdef FD_PROFILE_WAITS
    const long long t_start = clock64();
#endif

    if (threadIdx.x == 0) {
        for (int i = 0; i < C::STAGES; ++i) {
            ptx::mbar_init(&kfull[i], 1);
            ptx::mbar_init(&kempty[i], 1);
        }
        for (int i = 0; i < C::USTAGES; ++i) {
            ptx::mbar_init(&ufull[i], 1);
            ptx::mbar_init(&uempty[i], 2);   // both P.U issuers
        }
        ptx::mbar_init(qfull, 1);
        ptx::mbar_init(qempty, C::WIDE ? 1 : 2);   // both Q.K^T issuers (one for wide operands)
        for (int i = 0; i < NSB; ++i) {
            ptx::mbar_init(&sfull[i], 1);
            ptx::mbar_init(&sempty[i], 2);   // both P.U issuers
            ptx::mbar_init(&pfull[i], 4);   // the 4 warps of the warpgroup owning buffer i
        }
        for (int i = 0; i < NSB; ++i) ptx::mbar_init(&ofull[i], 2);   // both P.U issuers
        ptx::mbar_init(oempty, 4);          // the 4 warps of the warpgroup that read O
        for (int i = 0; i < 4; ++i) ptx::mbar_init(&done[i], 1);   // one per MMA issuer
        *abort = 0;
        for (int i = 0; i < BM; ++i) aseq[i] = 0;
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
    if (warp == UTMA_WARP && lane == 0) ptx::prefetch_tmap(&tmu);
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
                const int64_t rt = w.rt, jt = w.jt;
                if (rt != cur_rt) {
                    if (qcount > 0 && !FD_WAIT(0, qempty, (qcount - 1) & 1, abort, status, WAIT_LIMIT_NS)) break;
                    ptx::mbar_expect_tx(qfull, C::Q_BYTES);
                    for (int kb = 0; kb < KF; ++kb)
                        ptx::tma_load_2d(sQ + kb * BOX_BYTES, &tmq, qfull, kb * 64, (int)(rt * BM));
                    if (NW) ptx::tma_load_2d(sQ + KF * BOX_BYTES, &tmq_n, qfull, KF * 64, (int)(rt * BM));
                    cur_rt = rt;
                    ++qcount;
                }
                if (pacing) pacing = tc::pace(sc, w.s, jt, abort, paced);
                if constexpr (C::WIDE) {
                    // one box per ring slot, in column order
                    bool ok = true;
                    for (int kb = 0; kb < KF + (NW ? 1 : 0) && ok; ++kb) {
                        if (!FD_WAIT(1, &kempty[stage], kph ^ 1, abort, status, WAIT_LIMIT_NS)) { ok = false; break; }
                        uint8_t* st = sK + stage * C::STAGE_BYTES;
                        if (kb < KF) {
                            ptx::mbar_expect_tx(&kfull[stage], KBOX_BYTES);
                            ptx::tma_load_2d(st, &tmk, &kfull[stage], kb * 64, (int)(jt * BN));
                        } else {
                            ptx::mbar_expect_tx(&kfull[stage], BN * NW * 2);
                            ptx::tma_load_2d(st, &tmk_n, &kfull[stage], KF * 64, (int)(jt * BN));
                        }
                        if (++stage == C::STAGES) { stage = 0; kph ^= 1; }
                    }
                    if (!ok) break;
                } else {
                    if (!FD_WAIT(1, &kempty[stage], kph ^ 1, abort, status, WAIT_LIMIT_NS)) break;
                    uint8_t* st = sK + stage * C::STAGE_BYTES;
                    ptx::mbar_expect_tx(&kfull[stage], C::STAGE_BYTES);
                    for (int kb = 0; kb < KF; ++kb)
                        ptx::tma_load_2d(st + kb * KBOX_BYTES, &tmk, &kfull[stage], kb * 64, (int)(jt * BN));
                    if (NW) ptx::tma_load_2d(st + KF * KBOX_BYTES, &tmk_n, &kfull[stage], KF * 64, (int)(jt * BN));
                    if (++stage == C::STAGES) { stage = 0; kph ^= 1; }
                }
            }
        }
    } else if (warp == UTMA_WARP) {
        if (lane == 0) {
            int ustage = 0;
            uint32_t uph = 0;
            uint8_t* sU = base + C::U_OFF;
            for (Walk w(sc, cta); !w.done(); w.next()) {
                const int64_t jt = w.jt;
                // U_hi^T rows [0, RP), U_lo^T rows [RP, 2 RP) of the same map
                if (!FD_WAIT(2, &uempty[ustage], uph ^ 1, abort, status, WAIT_LIMIT_NS)) break;
                uint8_t* su = sU + ustage * C::USTAGE_BYTES;
                ptx::mbar_expect_tx(&ufull[ustage], C::USTAGE_BYTES);
                for (int part2 = 0; part2 < 2; ++part2)
                    for (int h = 0; h < 2; ++h)
                        ptx::tma_load_2d(su + (h * 2 + part2) * C::UT_BOX, &tmu, &ufull[ustage],
                                         (int)(jt * BN + h * 64), part2 * RP);
                if (++ustage == C::USTAGES) { ustage = 0; uph ^= 1; }
            }
        }
    } else if (warp == MMA_WARP || warp == MMA_WARP + 1) {
        // ---- Q.K^T issuers: warp MMA_WARP + q takes the tiles m = q (mod 2) ----
        if (lane == 0) {
            const int q = warp - MMA_WARP;
            const uint32_t q_base = ptx::smem_u32(sQ), k_base = ptx::smem_u32(sK);
            int stage = 0;
            uint32_t kph = 0, qcount = 0;
            int64_t cur_rt = -1;
            for (Walk w(sc, cta); !w.done() && !(C::WIDE && q == 1); w.next()) {
                const int64_t m = w.s, rt = w.rt;
                const int b = (int)(m % NSB);
                if (rt != cur_rt) {
                    if (!FD_WAIT(6, qfull, qcount & 1, abort, status, WAIT_LIMIT_NS)) break;
                    ++qcount;
                    cur_rt = rt;
                }
                if constexpr (C::WIDE) {
                    // one issuer, every tile; the key boxes arrive one per ring slot
                    if (!FD_WAIT(8, &sempty[b], (uint32_t)(((m / NSB) & 1) ^ 1), abort, status, WAIT_LIMIT_NS)) break;
                    bool ok = true;
                    int ks = 0;
                    for (int kb = 0; kb < KF + (NW ? 1 : 0); ++kb) {
                        if (!FD_WAIT(7, &kfull[stage], kph, abort, status, WAIT_LIMIT_NS)) { ok = false; break; }
                        ptx::tc_fence_after();
                        const uint32_t ka = k_base + stage * C::STAGE_BYTES;
                        if (kb < KF) {
#pragma unroll
                            for (int k4 = 0; k4 < 4; ++k4, ++ks)
                                ptx::umma_ss(tmem + b * BN, G::desc(q_base, BM, ks), ptx::sw128_kmajor_desc(ka + k4 * 32),
                                             idesc_qk, ks > 0);
                        } else {
                            for (int k2 = 0; k2 < NW / 16; ++k2, ++ks) {
                                const uint64_t bd = NW == 32 ? ptx::sw64_kmajor_desc(ka + k2 * 32)
                                                             : ptx::sw32_kmajor_desc(ka + k2 * 32);
                                ptx::umma_ss(tmem + b * BN, G::desc(q_base, BM, ks), bd, idesc_qk, ks > 0);
                            }
                        }
                        ptx::umma_commit(&kempty[stage]);
                        if (++stage == C::STAGES) { stage = 0; kph ^= 1; }
                    }
                    if (!ok) break;
                    ptx::umma_commit(&sfull[b]);
                    if (w.seg_last()) ptx::umma_commit(qempty);
                    continue;
                }
                if ((int)(m & 1) == q) {
                    if (!FD_WAIT(7, &kfull[stage], kph, abort, status, WAIT_LIMIT_NS)) break;
                    if (!FD_WAIT(8, &sempty[b], (uint32_t)(((m / NSB) & 1) ^ 1), abort, status, WAIT_LIMIT_NS)) break;
                    ptx::tc_fence_after();
                    const uint32_t ka = k_base + stage * C::STAGE_BYTES;
                    FD_SPAN_BEGIN;
#pragma unroll
                    for (int ks = 0; ks < G::KSTEPS; ++ks)
                        ptx::umma_ss(tmem + b * BN, G::desc(q_base, BM, ks), G::desc(ka, BN, ks), idesc_qk, ks > 0);
                    ptx::umma_commit(&sfull[b]);
                    ptx::umma_commit(&kempty[stage]);
                    FD_SPAN_END(14);
                }
                // both issuers arrive at every row-tile end (qempty counts 2)
                if (w.seg_last()) ptx::umma_commit(qempty);
                if (++stage == C::STAGES) { stage = 0; kph ^= 1; }
            }
            ptx::umma_commit(&done[q]);
            FD_WAIT(11, &done[q], 0, abort, status, WAIT_LIMIT_NS);
        }
    } else if (warp == PV_WARP0 || warp == PV_WARP1) {
        // ---- P.U issuers.  Three products (fp32-class tiles): warp PV_WARP0 runs
        //      O1 += P_hi [U_hi; U_lo] (N = 2 RP), warp PV_WARP1 O2 += P_lo U_hi
        //      (N = RP).  Two products (16-bit tiles, P rounded once to fp16):
        //      both run P [U_hi; U_lo], warp PV_WARP0 over keys 0-63 of the tile
        //      into O1, warp PV_WARP1 over keys 64-127 into O2.  Each
        //      tcgen05.mma costs its issuing thread ~100 cycles, so independent
        //      chains get their own issuing warps.
        if (lane == 0) {
            const int t = warp - PV_WARP0;
            const uint32_t u_base = ptx::smem_u32(base + C::U_OFF);
            const uint32_t idesc = (t == 0 || !three) ? idesc_pv2 : idesc_pv;
            const uint32_t dcol = tmem + O_COL + (t == 0 ? 0u : 2u * RP);
            const int ks0 = three ? 0 : t * (BN / 32), ks1 = three ? BN / 16 : ks0 + BN / 32;
            int ustage = 0;
            uint32_t uph = 0, ocount = 0;
            bool fresh = true;
            int gcnt = 0;
            for (Walk w(sc, cta); !w.done(); w.next()) {
                const int64_t m = w.s;
                const int pb = (int)(m % NSB);
                if (!FD_WAIT(3, &ufull[ustage], uph, abort, status, WAIT_LIMIT_NS)) break;
                if (!FD_WAIT(4, &pfull[pb], (uint32_t)((m / NSB) & 1), abort, status, WAIT_LIMIT_NS)) break;
                if (fresh && !FD_WAIT(5, oempty, (ocount & 1) ^ 1, abort, status, WAIT_LIMIT_NS)) break;
                ptx::tc_fence_after();
                const uint32_t ut = u_base + ustage * C::USTAGE_BYTES;
                FD_SPAN_BEGIN;
                for (int ks = ks0; ks < ks1; ++ks) {
                    // U_hi^T rows then U_lo^T rows of this 64-key box: one 2 RP-row operand
                    const uint32_t off = (ks >> 2) * 2 * C::UT_BOX + (ks & 3) * 32;
                    // keys 16ks..16ks+15: P (or P_hi) in 8 columns, P_lo in the next 8
                    const uint32_t a = tmem + pb * BN + ks * 16 + ((t == 0 || !three) ? 0u : 8u);
                    ptx::umma_ts(dcol, a, ptx::sw128_kmajor_desc(ut + off), idesc, (fresh && ks == ks0) ? 0u : 1u);
                }
                fresh = false;
                ptx::umma_commit(&sempty[pb]);
                ptx::umma_commit(&uempty[ustage]);
                FD_SPAN_END(13);
                if (++ustage == C::USTAGES) { ustage = 0; uph ^= 1; }
                const bool seg_last = w.seg_last();
                if (seg_last || ++gcnt == ogroup) {     // end of an O group
                    ptx::umma_commit(&ofull[pb]);       // the group's reader: tile m's warpgroup
                    fresh = true;
                    ++ocount;
                    gcnt = 0;
                }
            }
            ptx::umma_commit(&done[2 + t]);
            FD_WAIT(11, &done[2 + t], 0, abort, status, WAIT_LIMIT_NS);
        }
    } else {
        // ---- epilogue warpgroups ------------------------------------------
        // Warpgroup wg turns the S tiles m = wg (mod 3) into P.  At the end of an
        // O group the warpgroup that made the group's last P reads O (every
        // column) and adds it into the shared running sum of the segment
        // (sacc, [RP][BM] fp32); aseq[row] counts the groups added, so the next
        // group's reader (the thread of the same row in another warpgroup)
        // waits for it.  Each warpgroup waits on its own ofull barrier, once per
        // group it reads, so no barrier phase can be skipped.
        const int wg = warp >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
        float* sacc = (float*)(base + C::ACC_OFF);
        uint32_t ogroups = 0, oread = 0;
        int gcnt = 0;
        bool seg_fresh = true;
        bool alive = true;
        for (Walk w(sc, cta); !w.done() && alive; w.next()) {
            const int64_t m = w.s, rt = w.rt;
            const bool mine = (int)(m % NSB) == wg;
            if (mine) {
                const int b = wg;
                if (!FD_WAIT(9, &sfull[b], (uint32_t)((m / NSB) & 1), abort, status, WAIT_LIMIT_NS)) { alive = false; break; }
                ptx::tc_fence_after();
                // the whole tile: the 16 keys of chunk c come back as P_hi (8
                // columns) and P_lo (8 columns) over the same 16 S columns,
                // which this thread has read before it writes them
                const uint32_t tb = t_lane + b * BN;
                uint32_t va[16], vb[16], ph[8], pl[8];
                ptx::tmem_ld16(tb, va);
                ptx::tmem_wait_ld16(va);
                if (three) {
#pragma unroll 1
                    for (int c = 0; c < BN / 16; c += 2) {
                        ptx::tmem_ld16(tb + (c + 1) * 16, vb);
                        exp2_to_f16x2(va, ph, pl);
                        tmem_st8(tb + c * 16, ph);
                        tmem_st8(tb + c * 16 + 8, pl);
                        ptx::tmem_wait_ld16(vb);
                        if (c + 2 < BN / 16) ptx::tmem_ld16(tb + (c + 2) * 16, va);
                        exp2_to_f16x2(vb, ph, pl);
                        tmem_st8(tb + (c + 1) * 16, ph);
                        tmem_st8(tb + (c + 1) * 16 + 8, pl);
                        if (c + 2 < BN / 16) ptx::tmem_wait_ld16(va);
                    }
                } else {
#pragma unroll 1
                    for (int c = 0; c < BN / 16; c += 2) {
                        ptx::tmem_ld16(tb + (c + 1) * 16, vb);
                        exp2_to_f16(va, ph);
                        tmem_st8(tb + c * 16, ph);
                        ptx::tmem_wait_ld16(vb);
                        if (c + 2 < BN / 16) ptx::tmem_ld16(tb + (c + 2) * 16, va);
                        exp2_to_f16(vb, ph);
                        tmem_st8(tb + (c + 1) * 16, ph);
                        if (c + 2 < BN / 16) ptx::tmem_wait_ld16(va);
                    }
                }
                ptx::tmem_wait_st();
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(&pfull[b]);
            }
            const bool seg_last = w.seg_last();
            const bool grp_end = seg_last || (++gcnt == ogroup);
            if (!grp_end) continue;
            gcnt = 0;
            if (mine) {
                if (!FD_WAIT(10, &ofull[wg], oread & 1, abort, status, WAIT_LIMIT_NS)) { alive = false; break; }
                ++oread;
                if (!ptx::wait_seq(&aseq[row], ogroups, abort, status, WAIT_LIMIT_NS)) { alive = false; break; }
                ptx::tc_fence_after();
#pragma unroll
                for (int c16 = 0; c16 < RP; c16 += 16) {
                    // three products: P_hi U_hi, P_hi U_lo, P_lo U_hi; two: P U_hi and
                    // P U_lo over keys 0-63, then over keys 64-127
                    float o[16], t[16];
                    tmem_ld_cols<16>(t_lane + O_COL + c16, o);
                    tmem_ld_cols<16>(t_lane + O_COL + 2 * RP + c16, t);
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[i] += t[i];
                    tmem_ld_cols<16>(t_lane + O_COL + RP + c16, t);
                    if (!three) {
                        float t4[16];
                        tmem_ld_cols<16>(t_lane + O_COL + 3 * RP + c16, t4);
#pragma unroll
                        for (int i = 0; i < 16; ++i) t[i] += t4[i];
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float* a = &sacc[(c16 + i) * BM + row];
                        *a = seg_fresh ? o[i] + t[i] : *a + (o[i] + t[i]);
                    }
                }
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(oempty);
                if (seg_last) {
                    const int64_t gi = rt * BM + row;
                    const bool full = w.seg_full();
                    if (gi < nq) {
                        for (int c = 0; c < rc; ++c) {
                            const double val = (double)sacc[c * BM + row] * (double)colscale[c];
                            if (full) store_out(ep, gi, c, val);
                            else part[(((int64_t)cta * 2 + w.slot()) * BM + row) * RP + c] = val;
                        }
                    }
                }
                ptx::st_release_u32(&aseq[row], ogroups + 1);
            }
            ++ogroups;
            seg_fresh = seg_last;
        }
        ptx::tc_fence_before();
    }
    __syncthreads();
#ifdef FD_PROFILE_WAITS
    if (cta == 0 && threadIdx.x == 0) atomicAdd(&g_wait_cycles[15], (unsigned long long)(clock64() - t_start));
#endif
    if (warp == MMA_WARP) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// Sum the partials of row tiles cut between CTA ranges, in CTA order.
__global__ void tc_block_fixup_kernel(const double* __restrict__ part, Sched sc, int64_t nq, int rc, int rp,
                                      RowEpilogue ep) {
    const int64_t rt = blockIdx.x;
    for (int e = threadIdx.x; e < BM * rc; e += blockDim.x) {
        const int r = e / rc, col = e % rc;
        const int64_t gi = rt * BM + r;
        if (gi >= nq) continue;
        double sum = 0.0;
        const bool cut = for_each_cut_owner(sc, rt, [&](int c, int slot) {
            sum += part[(((int64_t)c * 2 + slot) * BM + r) * rp + col];
        });
        if (cut) store_out(ep, gi, col, sum);
    }
}

}  // namespace tcb

int block_rp(int rc) { return rc <= 16 ? 16 : (rc <= 32 ? 32 : 64); }

// cross-CTA partials, then one 256-byte line for the lockstep pacing counter
size_t tc_block_workspace_bytes(int rp) {
    return align256(sizeof(double) * 2 * (size_t)num_sms() * tcb::BM * rp) + 256;
}

struct BlockArgs {
    CUtensorMap mq, mk, mqn, mkn, mu;
    const float* colscale;
    int rc;
    int64_t nq;
    uint32_t iqk, ipv;
    tc::Sched sc;
    RowEpilogue ep;
    double* part;
    int ogroup;
    int three;
};

template <int KF, int NW, int RP>
static int launch_block_t(const BlockArgs& a, cudaStream_t s) {
    using C = tcb::Cfg<KF, NW, RP>;
    int* status = nullptr;
    FD_TRY(status_word(&status));
    FD_CUDA_TRY(cudaFuncSetAttribute(tcb::tc_block_kernel<KF, NW, RP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)C::SMEM_ALLOC));
    tcb::tc_block_kernel<KF, NW, RP><<<a.sc.grid, tcb::NTHREADS, C::SMEM_ALLOC, s>>>(
        a.mq, a.mk, a.mqn, a.mkn, a.mu, a.colscale, a.rc, a.nq, a.iqk, a.ipv, a.sc, a.ep, a.part, status,
        ptx::idesc_f32acc(tcb::BM, 2 * RP, true), a.ogroup, a.three);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

// Columns of U per launch: the accumulator blocks (4 x 32) fit next to the
// three 128-column S buffers in the 512 TMEM columns.
int block_max_cols(int d) { (void)d; return 32; }

// Process-wide block-path options (fd_set_block_options); 0 = the default.
static int g_block_group = 0;
static int g_block_products = 0;

// Key tiles per O accumulation group: 8 for the 16-bit tiles (bias 6e-6 against
// their 2e-3 error budget), 1 for the fp32-class tiles (bias 8e-7).
static int block_ogroup(int tile) {
    if (g_block_group > 0) return g_block_group;
    return tile == FD_TILE_F16X3 ? 1 : 8;
}

// Products per P.U: 3 (P_hi U_hi + P_hi U_lo + P_lo U_hi: P and U both to
// ~22 bits) by default.  2 rounds P once to fp16 for the 16-bit tiles
// (P U_hi + P U_lo, half the P.U instructions): about 2^-12 relative noise per
// kernel value, which a column whose sum cancels heavily can amplify past 2e-3.
static int block_products(int tile) {
    if (tile == FD_TILE_F16X3) return 3;
    return g_block_products == 2 ? 2 : 3;
}

template <int KF, int NW>
static int launch_block_kb(int rp, const BlockArgs& a, cudaStream_t s) {
    return rp == 16 ? launch_block_t<KF, NW, 16>(a, s) : launch_block_t<KF, NW, 32>(a, s);
}

// ut: [2 rp][ld] fp16 transposed, column-scaled right-hand side (hi rows, then
// lo rows); colscale: rp floats.
int launch_tc_block(const void* qop, int64_t nq, const void* kop, int64_t nk, int d, int tile, const void* ut,
                    int64_t ld, const float* colscale, int rc, const RowEpilogue& ep, void* ws, size_t ws_bytes,
                    cudaStream_t s) {
    if (nq == 0) return FD_OK;
    if (nk == 0) return launch_zero_rows(nq, rc, ep, s);
    FD_CHECK_ARG(rc >= 1 && rc <= 32, "block tile path: %d columns per launch (max 32)", rc);
    const int rp = block_rp(rc);
    const int kd = kd_tile(tile, d);
    int kf = 0, nw = 0;
    split_kd(kd, &kf, &nw);
    if (kd > 416) return set_error(FD_ERR_UNSUPPORTED, "tensor-core tile path: operand rows of %d columns (max 416)", kd);
    const size_t need = tc_block_workspace_bytes(rp);
    if (ws_bytes < need)
        return set_error(FD_ERR_WORKSPACE, "block tile path: workspace %zu B < %zu B", ws_bytes, need);
    const bool f16 = tile != FD_TILE_BF16;
    BlockArgs a;
    FD_TRY(make_tile_map(&a.mq, qop, nq, kd, tcb::BM, f16));
    FD_TRY(make_tile_map(&a.mk, kop, nk, kd, tcb::BN, f16));
    a.mqn = a.mq;
    a.mkn = a.mk;
    if (nw) {
        FD_TRY(make_tile_map(&a.mqn, qop, nq, kd, tcb::BM, f16, nw));
        FD_TRY(make_tile_map(&a.mkn, kop, nk, kd, tcb::BN, f16, nw));
    }
    FD_TRY(make_tile_map(&a.mu, ut, 2 * rp, ld, rp, true));   // U_hi^T rows then U_lo^T rows
    a.iqk = ptx::idesc_f32acc(tcb::BM, tcb::BN, f16);
    a.ipv = ptx::idesc_f32acc(tcb::BM, rp, true);
    a.sc = tc::Sched::make(cdiv(nq, tcb::BM), cdiv(nk, tcb::BN), num_sms(), (size_t)nk * kd * 2);
    a.part = (double*)ws;
    if (a.sc.full > 0) {
        a.sc.sync = (unsigned*)((uint8_t*)ws + need - 256);
        a.sc.pace_tiles = pace_tiles((size_t)tcb::BN * kd * 2 + (size_t)4 * tcb::BN * rp);
        FD_CUDA_TRY(cudaMemsetAsync(a.sc.sync, 0, sizeof(unsigned), s));
    }
    a.colscale = colscale;
    a.rc = rc;
    a.nq = nq;
    a.ep = ep;
    a.ogroup = block_ogroup(tile);
    a.three = block_products(tile) == 3;
    switch (kf * 100 + nw) {
        case 16: FD_TRY((launch_block_kb<0, 16>(rp, a, s))); break;
        case 32: FD_TRY((launch_block_kb<0, 32>(rp, a, s))); break;
        case 100: FD_TRY((launch_block_kb<1, 0>(rp, a, s))); break;
        case 116: FD_TRY((launch_block_kb<1, 16>(rp, a, s))); break;
        case 132: FD_TRY((launch_block_kb<1, 32>(rp, a, s))); break;
        case 200: FD_TRY((launch_block_kb<2, 0>(rp, a, s))); break;
        case 216: FD_TRY((launch_block_kb<2, 16>(rp, a, s))); break;
        case 232: FD_TRY((launch_block_kb<2, 32>(rp, a, s))); break;
        case 300: FD_TRY((launch_block_kb<3, 0>(rp, a, s))); break;
        case 316: FD_TRY((launch_block_kb<3, 16>(rp, a, s))); break;
        case 332: FD_TRY((launch_block_kb<3, 32>(rp, a, s))); break;
        case 400: FD_TRY((launch_block_kb<4, 0>(rp, a, s))); break;
        case 416: FD_TRY((launch_block_kb<4, 16>(rp, a, s))); break;
        case 432: FD_TRY((launch_block_kb<4, 32>(rp, a, s))); break;
        case 500: FD_TRY((launch_block_kb<5, 0>(rp, a, s))); break;
        case 516: FD_TRY((launch_block_kb<5, 16>(rp, a, s))); break;
        case 532: FD_TRY((launch_block_kb<5, 32>(rp, a, s))); break;
        case 600: FD_TRY((launch_block_kb<6, 0>(rp, a, s))); break;
        case 616: FD_TRY((launch_block_kb<6, 16>(rp, a, s))); break;
        case 632: FD_TRY((launch_block_kb<6, 32>(rp, a, s))); break;
        default: return set_error(FD_ERR_UNSUPPORTED, "block tile path: no kernel for kd=%d", kd);
    }
    tcb::tc_block_fixup_kernel<<<(unsigned)cdiv(nq, tcb::BM), 256, 0, s>>>(a.part, a.sc, nq, rc, rp, ep);
    FD_CUDA_TRY(cudaGetLastError());
    return FD_OK;
}

}  // namespace fd

extern "C" int fd_set_block_options(int group_tiles, int products) {
    if (group_tiles < 0 || group_tiles > 64)
        return fd::set_error(FD_ERR_ARG, "fd_set_block_options: group_tiles %d (0..64)", group_tiles);
    if (products != 0 && products != 2 && products != 3)
        return fd::set_error(FD_ERR_ARG, "fd_set_block_options: products %d (0, 2 or 3)", products);
    fd::g_block_group = group_tiles;
    fd::g_block_products = products;
    return FD_OK;
}

#ifdef FD_PROFILE_WAITS
// Read and clear the wait-time counters of the block kernel (profiling builds only).
extern "C" int fd_debug_wait_cycles(unsigned long long* host16) {
    FD_CUDA_TRY(cudaMemcpyFromSymbol(host16, fd::tcb::g_wait_cycles, 16 * sizeof(unsigned long long)));
    unsigned long long z[16] = {0};
    FD_CUDA_TRY(cudaMemcpyToSymbol(fd::tcb::g_wait_cycles, z, sizeof(z)));
    return FD_OK;
}
#endif
