// Pieces shared by the tcgen05 tile kernels (fd_tc.cu: r = 1, fd_tc_block.cu:
// block right-hand sides): the persistent work split and the two exp2 paths.
#pragma once
#include "fd_prep.cuh"
#include "fd_ptx.cuh"

namespace fd {
namespace tc {

// Column geometry of a tile operand in shared memory: KF full boxes of 64
// columns (128-byte rows, 128-byte swizzle), then an optional narrow box of
// NW in {0, 16, 32} columns (32- / 64-byte swizzle), so a row of kd = 64 KF + NW
// columns is stored without padding it to a multiple of 64.
template <int KF, int NW>
struct Geo {
    static constexpr int KSTEPS = KF * 4 + NW / 16;
    static constexpr uint32_t bytes(int rows) { return (uint32_t)rows * (KF * 128 + NW * 2); }
    // shared-memory descriptor of 16-column k-step ks of a tile of `rows` rows at saddr
    __device__ static __forceinline__ uint64_t desc(uint32_t saddr, int rows, int ks) {
        if (ks < KF * 4) return ptx::sw128_kmajor_desc(saddr + (ks >> 2) * rows * 128 + (ks & 3) * 32);
        const uint32_t nb = saddr + KF * rows * 128 + (ks - KF * 4) * 32;
        return NW == 32 ? ptx::sw64_kmajor_desc(nb) : ptx::sw32_kmajor_desc(nb);
    }
};

// Work split of the persistent kernels over (row tile, key tile) units.
//
// Contiguous mode (the key operand stays in L2): the units, row-major, are cut
// into grid contiguous ranges, one per CTA; a row tile cut between ranges
// leaves fp64 partials that the fix-up kernel sums in CTA order.
//
// Lockstep mode (a key operand larger than L2): first `full` whole row tiles per
// CTA, CTA c taking rows c, c + grid, ...: every CTA starts each of these rows at
// key tile 0 at about the same time, so the CTAs sweep K in near lockstep and a
// key tile is read from DRAM once per sweep and then served from L2 (with CTAs
// at scattered key offsets, a K larger than L2 is streamed from DRAM once per
// CTA).  The n_rem remaining row tiles (fewer than grid) are each cut into
// k = grid / n_rem key chunks: CTA c < k n_rem takes row c mod n_rem, chunk
// c / n_rem, so the CTAs of one chunk index again read the same key tiles
// together; the chunks' partials are summed by the fix-up in chunk order.
// Everything is deterministic.
struct Sched {
    int64_t n_jt;    // key tiles per row tile
    int64_t units;   // contiguous mode: units of the remainder region, (n_rt - full * grid) * n_jt
    int64_t full;    // whole row tiles per CTA (lockstep mode)
    int64_t n_rem;   // lockstep mode: remainder row tiles
    int k;           // lockstep mode: key chunks per remainder row (0 = contiguous mode)
    int grid;
    // pacing of the lockstep sweeps (see pace()): a zeroed global counter and
    // the key tiles per pacing chunk; null = no pacing
    unsigned* sync = nullptr;
    int64_t pace_tiles = 0;
    __host__ __device__ int64_t start(int c) const { return (int64_t)c * units / grid; }   // remainder range
    __host__ __device__ int64_t rem_rt0() const { return full * grid; }
    __host__ __device__ int64_t chunk0(int j) const { return (int64_t)j * n_jt / k; }
    // schedule for n_rt row tiles of n_jt key tiles on at most `sms` CTAs; the
    // lockstep mode only pays when the key operand does not stay in L2 anyway
    // (measured: +17 % at 288 MB of keys, through lower DRAM power and higher
    // clocks under the power cap; -3 % at 32 MB), so it starts above 48 MB
    static Sched make(int64_t n_rt, int64_t n_jt, int sms, size_t key_bytes) {
        Sched sc;
        sc.n_jt = n_jt;
        const int64_t total = n_rt * n_jt;
        sc.grid = (int)(total < sms ? total : sms);
        const bool lockstep = key_bytes > ((size_t)48 << 20) && n_jt >= sc.grid;
        sc.full = lockstep ? n_rt / sc.grid : 0;
        sc.n_rem = n_rt - sc.full * sc.grid;
        sc.k = (lockstep && sc.n_rem > 0) ? (int)(sc.grid / sc.n_rem) : 0;
        sc.units = sc.k ? 0 : sc.n_rem * n_jt;
        return sc;
    }
};

// Lockstep pacing.  The lockstep schedule only saves DRAM traffic while the
// CTAs sweeping K stay within the L2's reach of each other, and over ~100
// sweeps (configuration 5 at 2M points) they drift apart until every CTA
// streams K from DRAM (measured: 8.5 TB per launch, 3.4 TB/s, which lowers the
// power-capped clock).  So the key producer of every CTA, at the start of each
// chunk of pace_tiles key tiles of a whole-row sweep, counts itself in a global
// counter and waits until every CTA has started the chunk before: the CTAs
// then stay within about two chunks of each other.  The wait is a hint, not a
// barrier: it gives up after 1 ms (a CTA that is not resident yet cannot hold
// the others for longer; measured, giving up for good after one such wait let
// the sweeps drift apart again under the profiler) and returns false only when
// the kernel aborts, which ends the pacing of that producer.
// Called for the units a producer loads (every unit, or every other one);
// `last` (start at -1) remembers the chunk last counted.
__device__ __forceinline__ bool pace(const Sched& sc, int64_t s, int64_t jt, volatile int* abort, int64_t& last) {
    if (sc.sync == nullptr || s >= sc.full * sc.n_jt) return true;
    const int64_t nchunk = (sc.n_jt + sc.pace_tiles - 1) / sc.pace_tiles;
    const int64_t g = (s / sc.n_jt) * nchunk + jt / sc.pace_tiles;
    if (g == last) return true;
    last = g;
    atomicAdd(sc.sync, 1u);
    const uint64_t target = (uint64_t)sc.grid * (uint64_t)g;
    if (*(volatile unsigned*)sc.sync >= target) return true;
    const uint64_t t0 = ptx::globaltimer();
    while (*(volatile unsigned*)sc.sync < target) {
        if (*abort) return false;
        if (ptx::globaltimer() - t0 > 1000000ull) return true;
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 700
        __nanosleep(128);
#endif
    }
    return true;
}

// One CTA's units in processing order (the same sequence in every role).  The
// schedule's own fields are read from the kernel parameter, not copied, to keep
// the register count of the roles that carry a Walk down.
struct Walk {
    const Sched& sc;
    int64_t s = 0, steps, rt, jt, rem_first_rt, rem_jt0;
    __host__ __device__ Walk(const Sched& sc_, int c) : sc(sc_) {
        const int64_t rem_rt0 = sc.rem_rt0();
        if (sc.k > 0) {
            const bool busy = c < sc.k * sc.n_rem;
            const int j = busy ? (int)(c / sc.n_rem) : 0;
            rem_first_rt = rem_rt0 + (busy ? c % sc.n_rem : 0);
            rem_jt0 = sc.chunk0(j);
            steps = sc.full * sc.n_jt + (busy ? sc.chunk0(j + 1) - rem_jt0 : 0);
        } else {
            const int64_t u0 = sc.start(c);
            rem_first_rt = rem_rt0 + u0 / sc.n_jt;
            rem_jt0 = u0 - (rem_first_rt - rem_rt0) * sc.n_jt;
            steps = sc.full * sc.n_jt + sc.start(c + 1) - u0;
        }
        if (sc.full > 0) {
            rt = c;
            jt = 0;
        } else {
            rt = rem_first_rt;
            jt = rem_jt0;
        }
    }
    __host__ __device__ bool done() const { return s >= steps; }
    __host__ __device__ void next() {
        ++s;
        const int64_t nfull = sc.full * sc.n_jt;
        if (s == nfull) {
            rt = rem_first_rt;
            jt = rem_jt0;
        } else if (++jt == sc.n_jt) {
            jt = 0;
            rt += s < nfull ? sc.grid : 1;
        }
    }
    // last unit of this CTA's segment of row tile rt
    __host__ __device__ bool seg_last() const { return jt + 1 == sc.n_jt || s + 1 == steps; }
    // the segment covers all key tiles of the row (then the output is final)
    __host__ __device__ bool seg_full() const {
        const bool starts_at_0 = s < sc.full * sc.n_jt || rt != rem_first_rt || rem_jt0 == 0;
        return starts_at_0 && jt == sc.n_jt - 1;
    }
    // partial-sum slot of a cut row: 0 = the first remainder row, 1 = the last
    __host__ __device__ int slot() const { return rt == rem_first_rt ? 0 : 1; }
};

// Fix-up helper: calls f(c, slot) for every CTA holding a partial of row tile
// rt, in a fixed order; returns false (and calls nothing) when the row was not
// cut (its owner wrote it directly).
template <class F>
__host__ __device__ inline bool for_each_cut_owner(const Sched& sc, int64_t rt, F f) {
    if (rt < sc.rem_rt0()) return false;
    if (sc.k > 0) {
        if (sc.k == 1) return false;
        const int64_t r = rt - sc.rem_rt0();
        for (int j = 0; j < sc.k; ++j) f((int)(r + j * sc.n_rem), 0);
        return true;
    }
    const int64_t lo = (rt - sc.rem_rt0()) * sc.n_jt, hi = lo + sc.n_jt - 1;
    auto owner = [&](int64_t n) {
        int c = (int)(n * sc.grid / sc.units);
        if (c >= sc.grid) c = sc.grid - 1;
        while (c + 1 < sc.grid && sc.start(c + 1) <= n) ++c;
        while (c > 0 && sc.start(c) > n) --c;
        return c;
    };
    const int c_lo = owner(lo), c_hi = owner(hi);
    if (c_lo == c_hi) return false;
    for (int c = c_lo; c <= c_hi; ++c) {
        if (sc.start(c) == sc.start(c + 1)) continue;   // empty range
        f(c, (sc.rem_rt0() + sc.start(c) / sc.n_jt == rt) ? 0 : 1);
    }
    return true;
}

// ---- exp2 of a pair of exponents --------------------------------------------
// MUFU: two ex2.approx.ftz.  The exponent is <= 0 up to fp32 rounding of the
// exactly consistent packed operands, so no clamp at 0 is applied (the
// reference's clamp of d^2 at 0 only removes rounding noise).
__device__ __forceinline__ uint64_t exp2_mufu2(uint32_t a, uint32_t b) {
    return ptx::pack2(ptx::ex2_mufu(__uint_as_float(a)), ptx::ex2_mufu(__uint_as_float(b)));
}

// FMA pipe: 2^x = 2^j 2^f, j = round(x) by the 1.5*2^23 shift, f = x - j in
// [-1/2, 1/2], 2^f by a degree-4 polynomial (relative error 3.6e-6; fitted by
// the Remez exchange in tests/test_exp2_poly.py), 2^j added into the exponent
// field with one integer multiply-add.  x is clamped at -125 first so the
// exponent field cannot underflow.
__device__ __forceinline__ uint64_t exp2_poly2(uint32_t a, uint32_t b) {
    const float x0 = fmaxf(__uint_as_float(a), -125.0f);
    const float x1 = fmaxf(__uint_as_float(b), -125.0f);
    const uint64_t X = ptx::pack2(x0, x1);
    const uint64_t SH = ptx::pack2(12582912.0f, 12582912.0f);
    const uint64_t T = ptx::add2(X, SH);
    const uint64_t F = ptx::sub2(X, ptx::sub2(T, SH));
    uint64_t P = ptx::fma2(ptx::pack2(0.009782912f, 0.009782912f), F, ptx::pack2(0.055976883f, 0.055976883f));
    P = ptx::fma2(P, F, ptx::pack2(0.2402071f, 0.2402071f));
    P = ptx::fma2(P, F, ptx::pack2(0.6931136f, 0.6931136f));
    P = ptx::fma2(P, F, ptx::pack2(1.0f, 1.0f));
    uint32_t p0, p1, t0, t1;
    ptx::unpack2(P, p0, p1);
    ptx::unpack2(T, t0, t1);
    // the low 9 bits of the shifted value hold j mod 512, so t << 23 == j << 23 (mod 2^32)
    return ptx::pack2(__uint_as_float(p0 + (t0 << 23)), __uint_as_float(p1 + (t1 << 23)));
}

}  // namespace tc

// Host helpers defined in fd_tc.cu.
// 2-D map over a [rows][cols] 16-bit row-major matrix, box_cols x box_rows boxes
// with the swizzle that matches box_cols (64 -> 128 B, 32 -> 64 B, 16 -> 32 B).
int make_tile_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int box_rows, bool f16,
                  int box_cols = 64);
// kd = 64 kf + nw with nw in {0, 16, 32} (a remainder of 48 takes a full box).
void split_kd(int kd, int* kf, int* nw);
int num_sms();
// Key tiles per lockstep pacing chunk (about 8 MB) for a key tile of this many bytes (key operand + right-hand side).
int64_t pace_tiles(size_t bytes_per_key_tile);

}  // namespace fd
