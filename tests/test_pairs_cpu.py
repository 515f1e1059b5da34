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


def test_relay_pieces_pair_park_and_resume_byte_for_byte():
    """The e2e relay cuts every park segment and its resume twin at the same places: piece k of the park writes
    exactly the host bytes piece k of the resume reads, and together they cover the whole image."""
    kg = skv.KvGeometry()
    t = 32768 + 5

    class FakePool:                              # segments read only a pool's base address and block count
        base, n_blocks = 1 << 40, 4096

    src = skv.PooledSequence(kg, FakePool(), t, kg.n_qsa, None, 2 << 40, 3 << 40, 4 << 40)
    host = 5 << 40
    park = skv.pack_segments(src, host)
    resume = skv.unpack_segments(host, src)
    pieces = bench.relay_pieces(park, resume)
    assert len(pieces) > len(park)
    covered = 0
    for p, r in pieces:
        assert p.bytes == r.bytes and p.bytes <= bench.RELAY_CHUNK_BYTES
        assert p.dst == r.src                   # the park piece's host range is the resume piece's host range
        covered += p.bytes
    assert covered == sum(s.bytes for s in park)


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
        q.put((rank, checks, float(elapsed[0]), per.tolist(), res["value"]))
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
        rank, checks, elapsed, per, value = q.get(timeout=120)
        out[rank] = (checks, elapsed, per, value)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out[0][0] == {"handle": True, "tables": True}
    assert out[0][1] == out[1][1] == 11.0
    assert out[0][2] == [2.0, 2.0, 3.0]
    assert out[0][3] == pytest.approx(1 * 1000 * 3 / 0.011 / 1e9)
