// handoff_schedule.cpp - skv_schedule_phases: the port-exclusive order of a many-to-many hand-off batch, and
// skv_slice_segments: one run's share of its flow as segments (declared in include/strata_kv.h).  Host-only.
//
// D[s][d] = the bytes source s hands destination d.  No order ends before the busiest port (a row or column sum,
// M) has carried its load.  The order built here meets that bound when every port moves at one rate:
//   1. pad D with idle time until every row and column sums to M (north-west corner rule);
//   2. split the padded matrix into permutation phases (Birkhoff-von Neumann): a non-negative matrix whose rows
//      and columns share one sum always has a permutation of positive entries; take the one whose smallest entry
//      is largest, subtract that entry along it, repeat.  Every step empties at least one entry, so there are at
//      most n * n phases, and their weights add up to M;
//   3. cut each flow (s, d) at its phases' boundaries, real bytes first (a phase's share may end early: padding);
//   4. chain the readers of each source: a run from a source another destination read before waits for that
//      destination's signal.  Every wait points at an earlier phase, so the waits cannot form a cycle.
#include "strata_kv.h"
#include "skv_internal.h"

#include <algorithm>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace {

using Matrix = std::vector<std::vector<int64_t>>;

/// Largest-smallest-entry permutation by exhaustive search (n <= 6; ties go to the lexicographically largest).
std::vector<int> best_permutation_exhaustive(const Matrix& P, int64_t& best_w) {
    const int n = (int) P.size();
    std::vector<int> p(n), best;
    for (int i = 0; i < n; ++i) p[i] = i;
    best_w = -1;
    do {
        int64_t w = INT64_MAX;
        for (int s = 0; s < n; ++s) w = std::min(w, P[s][p[s]]);
        if (w >= best_w) {   // permutations come in increasing order: >= keeps the largest of a tie
            best_w = w;
            best = p;
        }
    } while (std::next_permutation(p.begin(), p.end()));
    return best;
}

/// A perfect matching of rows to columns over entries >= threshold, by augmenting paths (rows and columns tried
/// in index order); empty when there is none.
bool augment(int r, const Matrix& P, int64_t threshold, std::vector<int>& match_col, std::vector<char>& seen) {
    const int n = (int) P.size();
    for (int c = 0; c < n; ++c) {
        if (P[r][c] >= threshold && !seen[c]) {
            seen[c] = 1;
            if (match_col[c] < 0 || augment(match_col[c], P, threshold, match_col, seen)) {
                match_col[c] = r;
                return true;
            }
        }
    }
    return false;
}
std::vector<int> perfect_matching(const Matrix& P, int64_t threshold) {
    const int n = (int) P.size();
    std::vector<int> match_col(n, -1);
    for (int r = 0; r < n; ++r) {
        std::vector<char> seen(n, 0);
        if (!augment(r, P, threshold, match_col, seen)) return {};
    }
    std::vector<int> perm(n);
    for (int c = 0; c < n; ++c) perm[match_col[c]] = c;
    return perm;
}

/// Largest-smallest-entry permutation by a binary search over the distinct positive entries (n > 6).
std::vector<int> best_permutation_matching(const Matrix& P, int64_t& best_w) {
    std::vector<int64_t> values;
    for (const auto& row : P)
        for (int64_t v : row)
            if (v > 0) values.push_back(v);
    std::sort(values.begin(), values.end());
    values.erase(std::unique(values.begin(), values.end()), values.end());
    int lo = 0, hi = (int) values.size() - 1;
    std::vector<int> best;
    while (lo <= hi) {
        const int mid = (lo + hi) / 2;
        std::vector<int> perm = perfect_matching(P, values[mid]);
        if (perm.empty()) {
            hi = mid - 1;
        } else {
            best = std::move(perm);
            lo = mid + 1;
        }
    }
    best_w = 0;
    if (best.empty()) return best;
    best_w = INT64_MAX;
    for (int s = 0; s < (int) P.size(); ++s) best_w = std::min(best_w, P[s][best[s]]);
    return best;
}

}  // namespace

extern "C" int skv_schedule_phases(const uint64_t* demand, int n_src, int n_dst, skv_sched_run* runs, int max_runs,
                                   int* n_runs, uint64_t* bound_bytes, int* n_phases) {
    using skv::fail;
    if (!demand || !runs || !n_runs || !bound_bytes || !n_phases || n_src < 1 || n_dst < 1 || n_src > 64 ||
        n_dst > 64 || max_runs < 1)
        return fail(SKV_EINVAL, "skv_schedule_phases: bad arguments (1 <= n_src, n_dst <= 64, outputs non-null)");
    const int n = std::max(n_src, n_dst);
    Matrix D(n, std::vector<int64_t>(n, 0));
    for (int s = 0; s < n_src; ++s)
        for (int d = 0; d < n_dst; ++d) {
            const uint64_t b = demand[(size_t) s * n_dst + d];
            if (b > (uint64_t) INT64_MAX / 64)
                return fail(SKV_ERANGE, "skv_schedule_phases: a flow is too large (at most 2^57 bytes)");
            D[s][d] = (int64_t) b;
        }
    std::vector<int64_t> row(n, 0), col(n, 0);
    for (int s = 0; s < n; ++s)
        for (int d = 0; d < n; ++d) {
            row[s] += D[s][d];
            col[d] += D[s][d];
        }
    int64_t M = 0;
    for (int i = 0; i < n; ++i) M = std::max({M, row[i], col[i]});

    // 1. pad to equal row and column sums
    Matrix P = D;
    std::vector<int64_t> rdef(n), cdef(n);
    for (int i = 0; i < n; ++i) {
        rdef[i] = M - row[i];
        cdef[i] = M - col[i];
    }
    for (int i = 0, j = 0; i < n && j < n;) {
        const int64_t x = std::min(rdef[i], cdef[j]);
        P[i][j] += x;
        rdef[i] -= x;
        cdef[j] -= x;
        const bool next_i = rdef[i] == 0, next_j = cdef[j] == 0;
        i += next_i;
        j += next_j;
    }

    // 2. permutation phases
    std::vector<std::pair<std::vector<int>, int64_t>> phases;
    auto any = [&]() {
        for (const auto& r : P)
            for (int64_t v : r)
                if (v) return true;
        return false;
    };
    while (any()) {
        if ((int) phases.size() > n * n) return fail(SKV_EINVAL, "skv_schedule_phases: the phase split did not end");
        int64_t w = 0;
        std::vector<int> perm = n <= 6 ? best_permutation_exhaustive(P, w) : best_permutation_matching(P, w);
        if (perm.empty() || w <= 0)
            return fail(SKV_EINVAL, "skv_schedule_phases: no positive permutation (the padded matrix is not balanced)");
        for (int s = 0; s < n; ++s) P[s][perm[s]] -= w;
        phases.emplace_back(std::move(perm), w);
    }

    // 3 + 4. runs per destination, readers of each source chained
    Matrix left = D;
    Matrix cursor(n, std::vector<int64_t>(n, 0));
    std::vector<int> count(n_dst, 0);
    std::map<int, std::pair<int, int>> last;   // source -> (destination, run index) of its latest real run
    for (int k = 0; k < (int) phases.size(); ++k) {
        const auto& [perm, w] = phases[(size_t) k];
        for (int s = 0; s < n; ++s) {
            const int d = perm[s];
            const int64_t real = std::min(w, left[s][d]);
            if (real == 0) continue;   // padding (every real flow has s < n_src and d < n_dst)
            left[s][d] -= real;
            const int idx = count[d];
            if (idx >= max_runs)
                return fail(SKV_ERANGE, "skv_schedule_phases: a destination has more than max_runs runs");
            skv_sched_run& run = runs[(size_t) d * max_runs + idx];
            run.phase = k;
            run.src = s;
            run.lo = (uint64_t) cursor[s][d];
            run.hi = (uint64_t) (cursor[s][d] + real);
            run.wait = -1;
            run.signal_dst = -1;
            run.signal_idx = -1;
            run.reserved = 0;
            cursor[s][d] += real;
            auto it = last.find(s);
            if (it != last.end() && it->second.first != d) {
                run.wait = idx;
                skv_sched_run& prev = runs[(size_t) it->second.first * max_runs + it->second.second];
                prev.signal_dst = d;
                prev.signal_idx = idx;
            }
            last[s] = {d, idx};
            count[d] = idx + 1;
        }
    }
    for (int d = 0; d < n_dst; ++d) n_runs[d] = count[d];
    *bound_bytes = (uint64_t) M;
    *n_phases = (int) phases.size();
    return SKV_OK;
}

extern "C" int skv_slice_segments(const skv_segment* segs, int n_segs, uint64_t lo, uint64_t hi, skv_segment* out,
                                  int out_cap, int* n_out) {
    using skv::fail;
    if (n_segs < 0 || (n_segs && !segs) || out_cap < 0 || (out_cap && !out) || !n_out || hi < lo)
        return fail(SKV_EINVAL, "skv_slice_segments: bad arguments");
    int k = 0;
    uint64_t at = 0;
    for (int i = 0; i < n_segs; ++i) {
        const skv_segment& g = segs[i];
        const bool paged = g.src_pages || g.dst_pages;
        const uint64_t unit = paged ? g.page_bytes : 16;
        if (unit == 0 || g.bytes % unit)
            return fail(SKV_EINVAL, "skv_slice_segments: segment " + std::to_string(i) +
                                        " is not whole pages (paged) or 16-byte units (contiguous)");
        const uint64_t s_lo = std::max(lo, at), s_hi = std::min(hi, at + g.bytes);
        if (s_lo < s_hi) {
            const uint64_t a = (s_lo - at) / unit * unit;
            const uint64_t b = s_hi == at + g.bytes ? g.bytes : (s_hi - at) / unit * unit;
            if (a < b) {
                if (k >= out_cap) return fail(SKV_ERANGE, "skv_slice_segments: more pieces than out_cap");
                skv_segment& o = out[k++];
                o = g;
                const uint64_t first_page = paged ? a / unit : 0;
                if (!g.src_pages) o.src = static_cast<const uint8_t*>(g.src) + a;
                if (!g.dst_pages) o.dst = static_cast<uint8_t*>(g.dst) + a;
                if (g.src_pages) o.src_pages = g.src_pages + first_page;
                if (g.dst_pages) o.dst_pages = g.dst_pages + first_page;
                o.bytes = b - a;
            }
        }
        at += g.bytes;
    }
    *n_out = k;
    return SKV_OK;
}
