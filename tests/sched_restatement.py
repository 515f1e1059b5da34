"""A pure-Python restatement of skv_schedule_phases (csrc/host/handoff_schedule.cpp): TEST INFRASTRUCTURE.

The tests compare the library's native schedule against this one run for run; nothing outside tests/ imports it.
It also returns the phases themselves (permutation, weight), which the native call does not report.
"""
from __future__ import annotations

import itertools

import numpy as np


def _pad(D: np.ndarray) -> tuple:
    """The padded square matrix (every row and column summing to M) and M."""
    n = D.shape[0]
    M = int(max(D.sum(1).max(), D.sum(0).max())) if n else 0
    P = D.copy()
    rdef, cdef = M - P.sum(1), M - P.sum(0)
    i = j = 0
    while i < n and j < n:
        x = min(rdef[i], cdef[j])
        P[i, j] += x
        rdef[i] -= x
        cdef[j] -= x
        i += rdef[i] == 0
        j += cdef[j] == 0
    return P, M


def _perfect_matching(allowed: np.ndarray):
    """A perfect matching of the bipartite graph `allowed` (rows -> columns) by augmenting paths, or None."""
    n = allowed.shape[0]
    match_col = [-1] * n

    def augment(r, seen):
        for c in range(n):
            if allowed[r, c] and not seen[c]:
                seen[c] = True
                if match_col[c] < 0 or augment(match_col[c], seen):
                    match_col[c] = r
                    return True
        return False

    for r in range(n):
        if not augment(r, [False] * n):
            return None
    perm = [0] * n
    for c, r in enumerate(match_col):
        perm[r] = c
    return tuple(perm)


def _bottleneck_permutation(P: np.ndarray) -> tuple:
    """The permutation whose smallest entry is largest, and that entry.  Exhaustive (ties to the largest
    permutation in lexicographic order) up to 6 x 6; above, a binary search over thresholds with matchings."""
    n = P.shape[0]
    if n <= 6:
        w, perm = max((min(int(P[s, p[s]]) for s in range(n)), p) for p in itertools.permutations(range(n)))
        return perm, w
    values = np.unique(P[P > 0])
    lo, hi, best = 0, len(values) - 1, None
    while lo <= hi:
        mid = (lo + hi) // 2
        perm = _perfect_matching(P >= values[mid])
        if perm is None:
            hi = mid - 1
        else:
            best, lo = perm, mid + 1
    if best is None:
        return None, 0
    return best, min(int(P[s, best[s]]) for s in range(n))


def schedule(demand: dict, sources: list | None = None, destinations: list | None = None) -> dict:
    """The port-exclusive order of a batch of hand-offs.

    `demand` maps (source, destination) to bytes; `sources` and `destinations` fix the order of the matrix's rows
    and columns (default: sorted).  Returns {"bound_bytes": M, "phases": [(perm, w)], "runs": {destination:
    [run]}}: perm maps source index -> destination index (indices past the given lists are idle padding), and a
    run is {"phase", "src", "lo", "hi" (its byte range of the flow src -> destination), "wait" (this
    destination's flag index, or None), "signal" ((destination, flag index) to release after the run, or None)};
    a destination's flag index is its run index."""
    sources = list(sources) if sources is not None else sorted({s for s, _ in demand})
    destinations = list(destinations) if destinations is not None else sorted({d for _, d in demand})
    n = max(len(sources), len(destinations))
    D = np.zeros((n, n), dtype=np.int64)
    for (s, d), b in demand.items():
        if b < 0:
            raise ValueError("a flow cannot move a negative number of bytes")
        D[sources.index(s), destinations.index(d)] += int(b)
    P, M = _pad(D)
    phases = []
    while P.any():
        perm, w = _bottleneck_permutation(P)
        if w <= 0:
            raise RuntimeError("no positive permutation: the padded matrix is not balanced")
        phases.append((perm, w))
        for s in range(n):
            P[s, perm[s]] -= w
    left = D.copy()
    cursor = np.zeros((n, n), dtype=np.int64)
    runs = {d: [] for d in destinations}
    last = {}                                    # source -> (destination, run index) of its latest real run
    for k, (perm, w) in enumerate(phases):
        for s in range(n):
            d = perm[s]
            real = int(min(w, left[s, d]))
            if real == 0:
                continue
            left[s, d] -= real
            dst, src = destinations[d], sources[s]
            run = {"phase": k, "src": src, "lo": int(cursor[s, d]), "hi": int(cursor[s, d]) + real,
                   "wait": None, "signal": None}
            cursor[s, d] += real
            idx = len(runs[dst])
            prev = last.get(src)
            if prev is not None and prev[0] != dst:
                run["wait"] = idx
                runs[prev[0]][prev[1]]["signal"] = (dst, idx)
            runs[dst].append(run)
            last[src] = (dst, idx)
    return {"bound_bytes": M, "phases": phases, "runs": runs}
