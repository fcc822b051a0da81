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
// First `full` whole row tiles per CTA, CTA c taking rows c, c + grid, ...:
// every CTA starts each of these rows at key tile 0 at about the same time, so
// the CTAs sweep K in near lockstep and a key tile is read from DRAM once per
// sweep and then served from L2 (with CTAs at scattered key offsets, a K larger
// than L2 is streamed from DRAM once per CTA).  The remaining row tiles
// (fewer than grid) are cut into grid contiguous ranges of units; a row tile
// cut between ranges leaves fp64 partials that the fix-up kernel sums in CTA
// order (deterministic).
struct Sched {
    int64_t n_jt;    // key tiles per row tile
    int64_t units;   // units of the remainder region: (n_rt - full * grid) * n_jt
    int64_t full;    // whole row tiles per CTA
    int grid;
    __host__ __device__ int64_t start(int c) const { return (int64_t)c * units / grid; }   // remainder range
    __host__ __device__ int64_t rem_rt0() const { return full * grid; }
    // schedule for n_rt row tiles of n_jt key tiles on at most `sms` CTAs; the
    // lockstep rows only pay when the key operand does not stay in L2 anyway
    // (measured: +17 % at 288 MB of keys, through lower DRAM power and higher
    // clocks under the power cap; -3 % at 32 MB), so below `key_bytes` of
    // 48 MB every unit goes to the contiguous ranges
    static Sched make(int64_t n_rt, int64_t n_jt, int sms, size_t key_bytes) {
        Sched sc;
        sc.n_jt = n_jt;
        const int64_t total = n_rt * n_jt;
        sc.grid = (int)(total < sms ? total : sms);
        const bool lockstep = key_bytes > ((size_t)48 << 20);
        sc.full = (lockstep && n_rt >= sc.grid) ? n_rt / sc.grid : 0;
        sc.units = (n_rt - sc.full * sc.grid) * n_jt;
        return sc;
    }
};

// One CTA's units in processing order (the same sequence in every role).
struct Walk {
    int64_t s = 0, steps, nfull, rt, jt, rem_first_rt, rem_u0;
    int64_t n_jt, grid, rem_rt0;
    __device__ Walk(const Sched& sc, int c) {
        n_jt = sc.n_jt;
        grid = sc.grid;
        rem_rt0 = sc.rem_rt0();
        nfull = sc.full * sc.n_jt;
        rem_u0 = sc.start(c);
        steps = nfull + sc.start(c + 1) - rem_u0;
        rem_first_rt = rem_rt0 + rem_u0 / n_jt;
        if (nfull > 0) {
            rt = c;
            jt = 0;
        } else {
            rt = rem_first_rt;
            jt = rem_u0 - (rt - rem_rt0) * n_jt;
        }
    }
    __device__ bool done() const { return s >= steps; }
    __device__ void next() {
        ++s;
        if (s == nfull) {
            rt = rem_first_rt;
            jt = rem_u0 - (rt - rem_rt0) * n_jt;
        } else if (++jt == n_jt) {
            jt = 0;
            rt += s < nfull ? grid : 1;
        }
    }
    // last unit of this CTA's segment of row tile rt
    __device__ bool seg_last() const { return jt + 1 == n_jt || s + 1 == steps; }
    // the segment covers all key tiles of the row (then the output is final)
    __device__ bool seg_full() const {
        const bool starts_at_0 = s < nfull || rt != rem_first_rt || rem_u0 == (rt - rem_rt0) * n_jt;
        return starts_at_0 && jt == n_jt - 1;
    }
    // partial-sum slot of a cut row: 0 = the first remainder row, 1 = the last
    __device__ int slot() const { return rt == rem_first_rt ? 0 : 1; }
};

// Fix-up helper: the CTAs whose remainder ranges touch row tile rt
// (c_lo == c_hi: the row was not cut; whole rows are never cut).
__device__ inline void cut_owners(const Sched& sc, int64_t rt, int* c_lo, int* c_hi) {
    *c_lo = *c_hi = 0;
    if (rt < sc.rem_rt0()) return;
    const int64_t lo = (rt - sc.rem_rt0()) * sc.n_jt, hi = lo + sc.n_jt - 1;
    auto owner = [&](int64_t n) {
        int c = (int)(n * sc.grid / sc.units);
        if (c >= sc.grid) c = sc.grid - 1;
        while (c + 1 < sc.grid && sc.start(c + 1) <= n) ++c;
        while (c > 0 && sc.start(c) > n) --c;
        return c;
    };
    *c_lo = owner(lo);
    *c_hi = owner(hi);
}
// slot of CTA c's partial for row tile rt (c in [c_lo, c_hi], non-empty range)
__device__ inline int cut_slot(const Sched& sc, int c, int64_t rt) {
    return (sc.rem_rt0() + sc.start(c) / sc.n_jt == rt) ? 0 : 1;
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
// flashdiffusion_b200/csrc/exp2_poly_fit.py), 2^j added into the exponent
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

}  // namespace fd
