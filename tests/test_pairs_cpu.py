"""The N > 1 host logic of bench.py on CPU: pairing, the decode GPU's state-arena layout, the handle exchange and
the max-over-ranks reductions, run as world_size-2 `gloo` ranks (the GPU copies themselves are covered by the
GPU tests)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
import handoff_schedule
import sched_restatement
import skv


def test_pair_roles():
    assert [bench.pair_role(r, 2) for r in range(2)] == [("prefill", 1, True), ("decode", 0, True)]
    roles = [bench.pair_role(r, 8) for r in range(8)]
    assert [r[0] for r in roles] == ["prefill", "decode"] * 4
    assert all(roles[r][1] == r ^ 1 and roles[r][2] for r in range(8))
    assert bench.pair_role(2, 3) == ("prefill", 3, False)   # an unpaired last rank idles


def test_state_layout():
    kg = skv.KvGeometry()
    for t in (1, 5, 1024, 32768, 131071):
        lay = bench.state_layout(kg, t)
        assert lay["ids"] == kg.gdn_bytes
        assert lay["flag"] % 256 == 0 and lay["flag"] >= lay["ids"] + 4 * t
        assert lay["flag"] + 8 <= lay["bytes"] and lay["bytes"] % 1024 == 0


@pytest.mark.parametrize("ramp", [False, True])
def test_relay_pieces_pair_park_and_resume_byte_for_byte(ramp):
    """The e2e relay cuts the park segments and their resume twins at the same places: piece k of the park writes
    exactly the host bytes piece k of the resume reads, and together they cover the whole image in order.  With the
    ramp, the first and last pieces grade from 1/16 of a piece up and back down."""
    kg = skv.KvGeometry()
    t = 32768 + 5

    class FakePool:                              # segments read only a pool's base address and block count
        base, n_blocks = 1 << 40, 4096

    src = skv.PooledSequence(kg, FakePool(), t, kg.n_qsa, None, 2 << 40, 3 << 40, 4 << 40)
    host = 5 << 40
    park = skv.pack_segments(src, host)
    resume = skv.unpack_segments(host, src)
    pieces = bench.relay_pieces(park, resume, ramp=ramp)
    assert len(pieces) > len(park)
    covered, host_at, sizes = 0, [], []
    for pp, rp in pieces:
        assert len(pp) == len(rp)
        for p, r in zip(pp, rp):
            assert p.bytes == r.bytes
            assert p.dst == r.src               # the park piece's host range is the resume piece's host range
            host_at.append((p.dst, p.bytes))
        sizes.append(sum(p.bytes for p in pp))
        assert sizes[-1] <= bench.RELAY_CHUNK_BYTES
        covered += sizes[-1]
    assert covered == sum(s.bytes for s in park)
    # the host image is written front to back: each piece starts where the previous one ended or at a new segment
    assert len(set(host_at)) == len(host_at)
    if ramp:
        unit = bench.RELAY_CHUNK_BYTES // 16
        assert sizes[:5] == [unit, unit, 2 * unit, 4 * unit, 8 * unit] and sizes[-5:] == sizes[:5][::-1]


def test_mixed_plan_is_seeded_and_log_uniform():
    a, b = bench.mixed_plan(8, 1), bench.mixed_plan(8, 1)
    assert a == b and a != bench.mixed_plan(8, 2)
    lengths = np.asarray(a["lengths"])
    assert len(lengths) == bench.MIXED_SEQUENCES
    assert lengths.min() >= bench.MIXED_TOKENS[0] and lengths.max() <= bench.MIXED_TOKENS[1]
    assert set(a["owner"]) <= {0, 2, 4, 6} and set(a["target"]) <= {1, 3, 5, 7}
    # the log-uniform mean over [1K, 128K] is (128K - 1K) / ln 128 ~ 26.8K; many seeds stay near it
    means = [np.mean(bench.mixed_plan(8, s)["lengths"]) for s in range(40)]
    assert 20000 < np.mean(means) < 34000


def _play(sched, rate):
    """Run a phased schedule in an ideal model: a run starts when its GPU's previous run ended and, if it waits,
    when the run that signals it ended; it moves its bytes at `rate`.  Returns the makespan; fails on a deadlock."""
    runs = sched["runs"]
    signaller = {r["signal"]: (d, j) for d, rs in runs.items() for j, r in enumerate(rs) if r["signal"]}
    end, clock, at = {}, {d: 0.0 for d in runs}, {d: 0 for d in runs}
    moved = True
    while moved:
        moved = False
        for d, rs in runs.items():
            while at[d] < len(rs):
                j, r = at[d], rs[at[d]]
                start = clock[d]
                if r["wait"] is not None:
                    assert r["wait"] == j
                    dep = signaller[(d, j)]
                    if dep not in end:
                        break
                    start = max(start, end[dep])
                end[(d, j)] = clock[d] = start + (r["hi"] - r["lo"]) / rate
                at[d] += 1
                moved = True
    assert all(at[d] == len(rs) for d, rs in runs.items()), "deadlock"
    return max(clock.values())


@pytest.mark.parametrize("world,seed", [(8, 1), (8, 2), (8, 7), (4, 1), (4, 3), (2, 1)])
def test_phased_schedule_tiles_every_flow_and_meets_the_port_bound(world, seed):
    plan = bench.mixed_plan(world, seed)
    sizes = [24576 * t + 79036416 for t in plan["lengths"]]
    sched = bench.phased_schedule(plan, sizes, world)
    # the bound is the busiest port
    egress = {s: sum(b for b, o in zip(sizes, plan["owner"]) if o == s) for s in range(0, world, 2)}
    ingress = {d: sum(b for b, t in zip(sizes, plan["target"]) if t == d) for d in range(1, world, 2)}
    assert sched["bound_bytes"] == max(max(egress.values()), max(ingress.values()))
    # the native schedule equals the Python restatement run for run; its phases are permutations whose
    # weights sum to the bound
    ref = sched_restatement.schedule(bench.mixed_demand(plan, sizes), list(range(0, world, 2)),
                                     list(range(1, world, 2)))
    assert ref["runs"] == sched["runs"] and ref["bound_bytes"] == sched["bound_bytes"]
    assert len(ref["phases"]) == sched["n_phases"]
    assert sum(w for _, w in ref["phases"]) == sched["bound_bytes"]
    assert all(sorted(p) == list(range(world // 2)) for p, _ in ref["phases"])
    # every flow (src -> dst) is cut into consecutive byte ranges covering exactly its sequences
    for d, rs in sched["runs"].items():
        assert [r["phase"] for r in rs] == sorted(r["phase"] for r in rs)
        for s in range(0, world, 2):
            mine = [r for r in rs if r["src"] == s]
            want = sum(b for b, o, t in zip(sizes, plan["owner"], plan["target"]) if o == s and t == d)
            pos = 0
            for r in mine:
                assert r["lo"] == pos < r["hi"]
                pos = r["hi"]
            assert pos == want
    # in each phase a source feeds at most one decode GPU; reads of one source are chained by signals
    for k in range(sched["n_phases"]):
        srcs = [r["src"] for rs in sched["runs"].values() for r in rs if r["phase"] == k]
        assert len(srcs) == len(set(srcs))
    # with every port at one rate, the order ends exactly at the port bound (and never deadlocks)
    rate = 1e9
    assert _play(sched, rate) == pytest.approx(sched["bound_bytes"] / rate, rel=1e-9)


def test_port_bound_reports_the_busiest_port():
    plan = {"lengths": [1, 1, 1], "owner": [0, 0, 2], "target": [1, 3, 3]}
    b = bench.port_bound(plan, [100, 200, 300], 4)
    assert b["busiest_port_bytes"] == 500          # decode GPU 3's ingress
    assert b["ms"] == pytest.approx(500 / bench.NVLINK_PEER_COPY_GBS / 1e6, abs=1e-3)


def test_summarize_pairs():
    per = np.linspace(1.0, 2.0, 100)
    r = bench.summarize_pairs(150.0, per, pairs=4, seq_bytes=10 ** 9, steps=100)
    assert r["value"] == pytest.approx(4 * 100 * 1e9 / 0.150 / 1e9)
    assert r["per_pair_gbs"] == pytest.approx(1e9 / 0.0015 / 1e9)
    assert r["p50_ms"] == pytest.approx(1.5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        role, peer, active = bench.pair_role(rank, world)
        kg = skv.KvGeometry()
        mine = None
        if role == "decode":
            blocks = np.arange(kg.n_qsa * kg.blocks(1000), dtype=np.int32).reshape(kg.n_qsa, -1)[:, ::-1].copy()
            mine = {"pool": bytes([rank]) * 64, "state": bytes([rank + 100]) * 64,
                    "tables": skv.PooledSequence.host_tables(kg, blocks)}
        handles = [None] * world
        dist.all_gather_object(handles, mine)
        got = handles[peer]
        checks = {}
        if role == "prefill":
            checks["handle"] = got["pool"] == bytes([peer]) * 64 and got["state"] == bytes([peer + 100]) * 64
            checks["tables"] = got["tables"].shape == (kg.n_qsa, 2, kg.blocks(1000) * 64)
        elapsed = torch.tensor([10.0 + rank, 0.0])
        per = torch.tensor([1.0 + rank, 2.0, 3.0 - rank])
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        dist.all_reduce(per, op=dist.ReduceOp.MAX)
        res = bench.summarize_pairs(float(elapsed[0]), per.numpy(), world // 2, 1000, 3)
        # the per-pair verdicts and probe times as the bench gathers them: every rank's value, split by pair
        bench.device_align(torch, dist)   # every rank takes the same collective before a timed region
        mine_t = torch.tensor([float(rank == 1)])
        every = [torch.zeros_like(mine_t) for _ in range(world)]
        dist.all_gather(every, mine_t)
        pairs = bench.per_pair([float(e.item()) for e in every])
        q.put((rank, checks, float(elapsed[0]), per.tolist(), res["value"], pairs))
    finally:
        dist.destroy_process_group()


def test_two_rank_exchange_and_reductions():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in procs:
        rank, checks, elapsed, per, value, pairs = q.get(timeout=120)
        out[rank] = (checks, elapsed, per, value, pairs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out[0][0] == {"handle": True, "tables": True}
    assert out[0][1] == out[1][1] == 11.0
    assert out[0][2] == [2.0, 2.0, 3.0]
    assert out[0][3] == pytest.approx(1 * 1000 * 3 / 0.011 / 1e9)
    assert out[0][4] == out[1][4] == [(0.0, 1.0)]


def test_per_pair_split():
    assert bench.per_pair([1, 2, 3, 4, 5, 6, 7, 8]) == [(1, 2), (3, 4), (5, 6), (7, 8)]
    assert bench.per_pair([1, 2, 3]) == [(1, 2)]        # an unpaired last rank idles


def _fake_sequence_segments(kg, i, tokens):
    """Segments shaped like one pulled sequence (paged K/V per layer, contiguous GDN rows and ids) with made-up,
    distinct addresses: enough for the host-side cutting, nothing is launched."""
    n = kg.pages(tokens) * kg.page_bytes
    base = (i + 1) << 40
    segs = [skv.segment(base, base + (1 << 36), n, src_pages=base + (1 << 30) + 4096 * j,
                        dst_pages=base + (1 << 31) + 4096 * j, page_bytes=kg.page_bytes, src_page_limit=1 << 20,
                        dst_page_limit=1 << 20) for j in range(2 * kg.n_qsa)]
    segs.append(skv.segment(base + (1 << 37), base + (1 << 38), kg.gdn_bytes))
    segs.append(skv.segment(base + (1 << 39), base + (1 << 39) + (1 << 34), 16 * ((4 * tokens + 15) // 16)))
    return segs


def _merged(segs):
    """A list of segments with every piece that continues the one before it (same bases, the next table entry or
    the next address on each side) folded into it: pieces cut from one segment fold back into that segment."""
    out = []
    for g in segs:
        unit = g.page_bytes if (g.src_pages or g.dst_pages) else 16
        cur = [g.src, g.dst, g.src_pages, g.dst_pages, g.bytes, unit]
        if out:
            p = out[-1]
            n = p[4] // p[5]
            follows = (p[5] == unit and
                       (p[2] and cur[2] == p[2] + 4 * n and cur[0] == p[0] or not p[2] and not cur[2] and cur[0] == (p[0] or 0) + p[4]) and
                       (p[3] and cur[3] == p[3] + 4 * n and cur[1] == p[1] or not p[3] and not cur[3] and cur[1] == (p[1] or 0) + p[4]))
            if follows:
                p[4] += g.bytes
                continue
        out.append(cur)
    return out


@pytest.mark.parametrize("world,seed", [(8, 1), (8, 5), (4, 2)])
def test_phase_runs_move_every_sequence_once_in_schedule_order(world, seed):
    """What each decode GPU launches under the phased order: its runs' pieces, flow by flow, are exactly its
    sequences' segments (shortest first), every byte once; every sequence starts and ends in one run."""
    kg = skv.KvGeometry()
    plan = bench.mixed_plan(world, seed)
    sizes = [2 * kg.n_qsa * kg.pages(t) * kg.page_bytes + kg.gdn_bytes + 16 * ((4 * t + 15) // 16)
             for t in plan["lengths"]]
    for d in range(1, world, 2):
        mine = [i for i in range(len(sizes)) if plan["target"][i] == d]
        segs_of = {i: _fake_sequence_segments(kg, i, plan["lengths"][i]) for i in mine}
        runs = bench.phase_runs(d, plan, sizes, segs_of, world)
        for s in range(0, world, 2):
            flow = sorted((i for i in mine if plan["owner"][i] == s), key=lambda i: (plan["lengths"][i], i))
            want = _merged([seg for i in flow for seg in segs_of[i]])
            got = _merged([seg for r in runs if r["src"] == s for seg in r["pieces"]])
            assert got == want
        starts = [i for r in runs for i in r["starts"]]
        ends = [i for r in runs for i in r["ends"]]
        assert sorted(starts) == sorted(mine) == sorted(ends)
        where = {i: j for j, r in enumerate(runs) for i in r["ends"]}
        assert all(min(j for j, r in enumerate(runs) if i in r["starts"]) <= where[i] for i in mine)


def test_phase_runs_refuse_segments_that_disagree_with_the_sizes():
    kg = skv.KvGeometry()
    plan = bench.mixed_plan(4, 1)
    sizes = [2 * kg.n_qsa * kg.pages(t) * kg.page_bytes + kg.gdn_bytes + 16 * ((4 * t + 15) // 16)
             for t in plan["lengths"]]
    i = next(i for i in range(len(sizes)) if plan["target"][i] == 1)
    segs = _fake_sequence_segments(kg, i, plan["lengths"][i])[:-1]      # the ids segment left out
    with pytest.raises(ValueError):
        bench.phase_runs(1, plan, sizes, {i: segs}, 4)


def test_phase_summary_spans_and_rates():
    """Config 5's per-phase record: bytes summed over the decode GPUs, the span from the earliest start to the
    latest end, the aggregate rate over it, and the slowest run's own rate."""
    tl = [[[0.0, 1.0, 770_000_000, 0, 0, False], [1.1, 2.0, 700_000_000, 2, 1, True]],
          [[0.05, 1.05, 760_000_000, 2, 0, False], [1.2, 1.9, 100_000_000, 0, 1, True]]]
    p0, p1 = bench.phase_summary(tl)
    assert (p0["phase"], p0["runs"], p0["bytes"], p0["span_ms"]) == (0, 2, 1_530_000_000, 1.05)
    assert p0["gbs"] == pytest.approx(1_530_000_000 / 1.05e-3 / 1e9, abs=0.1)
    assert p0["slowest_run_gbs"] == pytest.approx(760.0)
    assert p1["span_ms"] == pytest.approx(0.9) and p1["slowest_run_gbs"] == pytest.approx(100_000_000 / 0.7e-3 / 1e9, abs=0.1)


@pytest.mark.parametrize("world,seed", [(8, 1), (8, 5), (8, 9), (4, 2)])
def test_fused_runs_move_the_same_bytes_with_the_same_hand_overs(world, seed):
    """Fusing back-to-back runs from one source (no flag between them) changes only the number of launches: each
    flow's pieces are the same in the same order, every wait and every signal survives exactly once, and no two
    neighbouring fused runs could be fused further."""
    kg = skv.KvGeometry()
    plan = bench.mixed_plan(world, seed)
    sizes = [2 * kg.n_qsa * kg.pages(t) * kg.page_bytes + kg.gdn_bytes + 16 * ((4 * t + 15) // 16)
             for t in plan["lengths"]]
    fused_any = False
    for d in range(1, world, 2):
        mine = [i for i in range(len(sizes)) if plan["target"][i] == d]
        segs_of = {i: _fake_sequence_segments(kg, i, plan["lengths"][i]) for i in mine}
        runs = bench.phase_runs(d, plan, sizes, segs_of, world)
        fused = handoff_schedule.fuse_runs(runs)
        fused_any = fused_any or len(fused) < len(runs)
        for s in range(0, world, 2):
            want = _merged([seg for r in runs if r["src"] == s for seg in r["pieces"]])
            got = _merged([seg for r in fused if r["src"] == s for seg in r["pieces"]])
            assert got == want
        assert sorted(r["wait"] for r in fused if r["wait"] is not None) == \
            sorted(r["wait"] for r in runs if r["wait"] is not None)
        assert sorted(r["signal"] for r in fused if r["signal"] is not None) == \
            sorted(r["signal"] for r in runs if r["signal"] is not None)
        assert sorted(i for r in fused for i in r["starts"]) == sorted(i for r in runs for i in r["starts"])
        assert sum(r.get("fused", 1) for r in fused) == len(runs)
        for a, b in zip(fused, fused[1:]):
            assert not (a["src"] == b["src"] and a["signal"] is None and b["wait"] is None)
    assert fused_any or world == 4


@pytest.mark.parametrize("world,seed", [(8, 1), (8, 5), (8, 9), (4, 2)])
def test_tail_phases_are_a_suffix_no_exclusive_run_waits_on(world, seed):
    """phased-tail drops the hand-overs of the last, small phases.  That is safe only if no run before the tail
    waits for a signal that a tail run sends: every run's wait is released by a run of an earlier phase."""
    kg = skv.KvGeometry()
    plan = bench.mixed_plan(world, seed)
    sizes = [2 * kg.n_qsa * kg.pages(t) * kg.page_bytes + kg.gdn_bytes + 16 * ((4 * t + 15) // 16)
             for t in plan["lengths"]]
    sched = bench.phased_schedule(plan, sizes, world)
    start = bench.tail_start(sched)
    phases = sorted({r["phase"] for runs in sched["runs"].values() for r in runs})
    if start is None:
        return
    assert start in phases and all(p >= start for p in phases[phases.index(start):])
    big = max(r["hi"] - r["lo"] for runs in sched["runs"].values() for r in runs if r["phase"] >= start)
    assert big < bench.TAIL_FRAC * sched["bound_bytes"]
    releaser = {}
    for d, runs in sched["runs"].items():
        for r in runs:
            if r["signal"] is not None:
                releaser[r["signal"]] = r["phase"]
    for d, runs in sched["runs"].items():
        for r in runs:
            if r["wait"] is not None:
                assert releaser[(d, r["wait"])] < r["phase"]
                if r["phase"] < start:
                    assert releaser[(d, r["wait"])] < start


class _RecordingLib:
    """Stands in for the C ABI: records every launch call and succeeds."""

    def __init__(self):
        self.calls = []

    def __getattr__(self, name):
        def call(*a):
            self.calls.append((name, a))
            return 0
        return call


@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("n_arrays", [1, 2, 3])
@pytest.mark.parametrize("wait,done", [(None, None), (0x1000, None), (None, 0x2000), (0x1000, 0x2000)])
def test_phase_run_launches(gated, n_arrays, wait, done):
    """A config-5 run waits for its hand-over before its first byte moves and releases the next reader only after
    its last copy: as launches of their own around the copies, or (gated) inside the first and last copy launch.
    Every array is copied exactly once, in order, on the run's stream, with the step's flag value."""
    L, marks = _RecordingLib(), []
    arrays = [(f"arr{q}", 10 + q) for q in range(n_arrays)]
    bench.issue_phase_run(L, arrays, wait, done, 7, "sp", gated, lambda: marks.append(len(L.calls)),
                          lambda: marks.append(len(L.calls)))
    names = [c[0] for c in L.calls]
    copied = [c[1][0] for c in L.calls if c[0] in ("skv_copy", "skv_copy_gated")]
    assert copied == [a for a, _ in arrays]
    assert all(c[1][-1] == "sp" for c in L.calls)
    if gated:
        assert "skv_wait_flag" not in names and "skv_signal" not in names
        gates = [(c[1][2], c[1][5]) for c in L.calls if c[0] == "skv_copy_gated"]
        expect = [(wait if q == 0 else None, done if q == n_arrays - 1 else None) for q in range(n_arrays)]
        assert gates == [g for g in expect if g != (None, None)]
        assert all(c[1][3] == 7 and c[1][6] == 7 and c[1][4] == bench.HANDOVER_WAIT_NS
                   for c in L.calls if c[0] == "skv_copy_gated")
        assert len(L.calls) == n_arrays and marks == [0, n_arrays]
    else:
        assert "skv_copy_gated" not in names
        assert names == (["skv_wait_flag"] if wait else []) + ["skv_copy"] * n_arrays + (["skv_signal"] if done else [])
        if wait:
            assert L.calls[0][1] == (wait, 7, bench.HANDOVER_WAIT_NS, "sp")
        if done:
            assert L.calls[-1][1] == (done, 7, "sp")
        assert marks == [int(bool(wait)), int(bool(wait)) + n_arrays]
