"""handoff_schedule / skv_schedule_phases: the port-exclusive order of many-to-many hand-offs (host-side policy),
on CPU, checked run for run against the Python restatement in tests/sched_restatement.py.

For any demand matrix - square or not, small (exhaustive permutation search) or large (bottleneck matchings) -
the phases add up to the busiest port's bytes, no source or destination carries two transfers in one phase,
every flow is cut into consecutive ranges covering exactly its bytes, the hand-over signals chain the readers of
each source, and played with every port at one rate the order ends exactly at the port bound without deadlock.
"""
import numpy as np
import pytest

import handoff_schedule as hs
import sched_restatement
import skv
from test_pairs_cpu import _play


def _check(demand, sched):
    ref = sched_restatement.schedule(demand)
    assert ref["runs"] == sched["runs"] and ref["bound_bytes"] == sched["bound_bytes"]
    assert len(ref["phases"]) == sched["n_phases"]
    rows, cols = {}, {}
    for (s, d), b in demand.items():
        rows[s] = rows.get(s, 0) + b
        cols[d] = cols.get(d, 0) + b
    M = max(list(rows.values()) + list(cols.values()))
    assert sched["bound_bytes"] == M
    assert sum(w for _, w in ref["phases"]) == M
    for perm, _ in ref["phases"]:
        assert sorted(perm) == list(range(len(perm)))
    for k in range(sched["n_phases"]):
        used = [(r["src"], d) for d, rs in sched["runs"].items() for r in rs if r["phase"] == k]
        assert len({s for s, _ in used}) == len(used) and len({d for _, d in used}) == len(used)
    for (s, d), b in demand.items():
        pos = 0
        for r in (r for r in sched["runs"][d] if r["src"] == s):
            assert r["lo"] == pos < r["hi"]
            pos = r["hi"]
        assert pos == b
    # every wait has exactly one signal pointing at it
    signals = [r["signal"] for rs in sched["runs"].values() for r in rs if r["signal"]]
    waits = [(d, r["wait"]) for d, rs in sched["runs"].items() for r in rs if r["wait"] is not None]
    assert sorted(signals) == sorted(waits)
    assert _play(sched, 1e9) == pytest.approx(M / 1e9, rel=1e-9)


@pytest.mark.parametrize("n_src,n_dst,seed", [(4, 4, 0), (3, 2, 1), (2, 5, 2), (1, 3, 3), (7, 7, 4), (8, 8, 5),
                                              (8, 3, 6), (10, 10, 7)])
def test_schedule_meets_the_port_bound(n_src, n_dst, seed):
    rng = np.random.default_rng(seed)
    demand = {}
    for s in range(n_src):
        for d in range(n_dst):
            if rng.random() < 0.7:
                demand[(f"p{s}", f"d{d}")] = int(rng.integers(1, 10 ** 9))
    if not demand:
        demand[("p0", "d0")] = 1
    sched = hs.schedule(demand)
    _check(demand, sched)


def test_one_hot_demand_is_one_phase():
    demand = {(0, 1): 100, (2, 3): 100}
    sched = hs.schedule(demand)
    assert sched["n_phases"] == 1
    assert all(r["wait"] is None and r["signal"] is None for rs in sched["runs"].values() for r in rs)


def test_launch_list_cuts_flows_and_refuses_a_mismatch():
    demand = {("a", "x"): 4096 * 6, ("b", "x"): 4096 * 2}
    sched = hs.schedule(demand)
    seg = lambda base, pages: skv.segment(base, base + (1 << 30), 4096 * pages, src_pages=base + 8,  # noqa: E731
                                          dst_pages=base + 16, page_bytes=4096, src_page_limit=99,
                                          dst_page_limit=99)
    flows = {"a": [("s1", [seg(1 << 32, 2)]), ("s2", [seg(2 << 32, 4)])], "b": [("s3", [seg(3 << 32, 2)])]}
    runs = hs.launch_list(sched, "x", flows)
    assert sum(g.bytes for r in runs for g in r["pieces"]) == 4096 * 8
    assert sorted(k for r in runs for k in r["ends"]) == ["s1", "s2", "s3"]
    with pytest.raises(ValueError):
        hs.launch_list(sched, "x", {"a": [("s1", [seg(1 << 32, 2)])], "b": flows["b"]})


def test_port_bound():
    b = hs.port_bound({(0, 1): 300, (0, 3): 200, (2, 3): 400}, 100.0)
    assert b["busiest_port_bytes"] == 600          # destination 3's ingress
    assert b["ms"] == pytest.approx(600 / 100.0 / 1e6, abs=1e-3)


def test_native_schedule_equals_the_restatement_on_random_batches():
    rng = np.random.default_rng(11)
    for trial in range(300):
        ns, nd = int(rng.integers(1, 10)), int(rng.integers(1, 10))
        demand = {(s, d): int(rng.integers(0, 1 << int(rng.integers(1, 40))))
                  for s in range(ns) for d in range(nd) if rng.random() < 0.6}
        if not any(demand.values()):
            continue
        got, ref = hs.schedule(demand), sched_restatement.schedule(demand)
        assert got["runs"] == ref["runs"] and got["bound_bytes"] == ref["bound_bytes"], trial
        assert got["n_phases"] == len(ref["phases"])


def test_native_schedule_refuses_bad_arguments():
    import ctypes as C
    L = skv.lib()
    runs = (skv.SchedRun * 4)()
    n_runs = (C.c_int * 2)()
    bound, phases = C.c_uint64(), C.c_int()
    demand = (C.c_uint64 * 4)(5, 0, 0, 5)
    assert L.skv_schedule_phases(demand, 0, 2, runs, 2, n_runs, C.byref(bound), C.byref(phases)) == skv.EINVAL
    assert L.skv_schedule_phases(demand, 2, 2, None, 2, n_runs, C.byref(bound), C.byref(phases)) == skv.EINVAL
    huge = (C.c_uint64 * 4)(1 << 62, 0, 0, 1)
    assert L.skv_schedule_phases(huge, 2, 2, runs, 2, n_runs, C.byref(bound), C.byref(phases)) == skv.ERANGE
    # destination 0 reads two sources, so it needs two runs; room for one is refused
    crowded = (C.c_uint64 * 4)(3, 0, 4, 0)
    assert L.skv_schedule_phases(crowded, 2, 2, runs, 1, n_runs, C.byref(bound), C.byref(phases)) == skv.ERANGE
    assert L.skv_schedule_phases(demand, 2, 2, runs, 2, n_runs, C.byref(bound), C.byref(phases)) == skv.OK
    assert bound.value == 5 and phases.value == 1 and list(n_runs) == [1, 1]
