// Host-side check of the persistent-kernel schedule (Sched / Walk /
// for_each_cut_owner of flashdiffusion_b200/csrc/fd_tc_common.cuh): for many
// shapes, every (row tile, key tile) unit is visited exactly once, every row
// tile is either written whole by one CTA or cut into partials whose
// (CTA, slot) pairs are unique and are exactly the owners the fix-up sums.
// Built and run by tests/test_schedule_cpu.py (nvcc, no GPU needed).
#include <cstdio>
#include <map>
#include <set>
#include <tuple>
#include <vector>

#include "../flashdiffusion_b200/csrc/fd_tc_common.cuh"

using fd::tc::Sched;
using fd::tc::Walk;

static int check(int64_t n_rt, int64_t n_jt, int sms, size_t key_bytes) {
    const Sched sc = Sched::make(n_rt, n_jt, sms, key_bytes);
    std::vector<int> seen((size_t)(n_rt * n_jt), 0);
    std::map<int64_t, int> whole;                                  // row -> writers of the whole row
    std::map<int64_t, std::set<std::pair<int, int>>> partial;      // row -> (cta, slot)
    std::set<std::pair<int, int>> slots_used;
    for (int c = 0; c < sc.grid; ++c) {
        int64_t seg_start_jt = -1;
        for (Walk w(sc, c); !w.done(); w.next()) {
            if (w.rt < 0 || w.rt >= n_rt || w.jt < 0 || w.jt >= n_jt) {
                printf("FAIL unit out of range rt=%lld jt=%lld\n", (long long)w.rt, (long long)w.jt);
                return 1;
            }
            seen[(size_t)(w.rt * n_jt + w.jt)] += 1;
            if (seg_start_jt < 0) seg_start_jt = w.jt;
            if (w.seg_last()) {
                if (w.seg_full()) {
                    if (seg_start_jt != 0 || w.jt != n_jt - 1) { printf("FAIL seg_full on a cut segment\n"); return 1; }
                    whole[w.rt] += 1;
                } else {
                    if (!slots_used.insert({c, w.slot()}).second) { printf("FAIL slot reused c=%d\n", c); return 1; }
                    partial[w.rt].insert({c, w.slot()});
                }
                seg_start_jt = -1;
            }
        }
    }
    for (size_t i = 0; i < seen.size(); ++i)
        if (seen[i] != 1) { printf("FAIL unit %zu seen %d times\n", i, seen[i]); return 1; }
    for (int64_t rt = 0; rt < n_rt; ++rt) {
        std::set<std::pair<int, int>> owners;
        const bool cut = fd::tc::for_each_cut_owner(sc, rt, [&](int c, int slot) { owners.insert({c, slot}); });
        const int w = whole.count(rt) ? whole[rt] : 0;
        if (cut) {
            if (w != 0 || owners != partial[rt]) { printf("FAIL row %lld: fix-up owners differ\n", (long long)rt); return 1; }
        } else if (w != 1 || !partial[rt].empty()) {
            printf("FAIL row %lld: not cut but written %d times\n", (long long)rt, w);
            return 1;
        }
    }
    return 0;
}

int main() {
    const size_t small = 1u << 20, big = (size_t)1 << 30;
    const int sms[] = {148, 132, 7, 1};
    const int64_t rts[] = {1, 2, 5, 147, 148, 149, 300, 781, 1954, 3907};
    const int64_t jts[] = {1, 3, 148, 150, 1563, 7813};
    int fails = 0, cases = 0;
    for (int g : sms)
        for (int64_t r : rts)
            for (int64_t j : jts)
                for (size_t kb : {small, big}) {
                    if (r * j > 4000000) continue;
                    ++cases;
                    if (check(r, j, g, kb)) {
                        printf("  case n_rt=%lld n_jt=%lld sms=%d key_bytes=%zu\n", (long long)r, (long long)j, g, kb);
                        ++fails;
                    }
                }
    if (fails) return 1;
    printf("OK %d cases\n", cases);
    return 0;
}
