"""Pin the oracle (oracle/kv_oracle.c + oracle/sr4h.py) before trusting it.

Two anchors, both the reference's own behaviour:
  * the golden fixtures in tests/golden/ (payloads and hashes written by the reference's
    conversation_snapshot_save + conversation_wire_encode, tests/golden/make_golden.py);
  * when oracle/_ref/libstrata_ref.so is present (built from the reference sources by oracle/Makefile),
    the live reference on fresh seeds and shapes.
"""
import json
import os

import numpy as np
import pytest

import oracle as O
import sr4h

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
with open(os.path.join(GOLDEN, "golden.json")) as f:
    G = json.load(f)
SMALL = O.Geometry(**G["small_geometry"])
needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built (no reference tree here)")


def payload(t):
    with open(os.path.join(GOLDEN, f"ref_payload_T{t}.bin"), "rb") as f:
        return f.read()


def oracle_image(g, s, tokens):
    """The SavedConversation the reference's save produces, built from the oracle's layout rules
    (conversation_snapshot.cpp:27-67, conversation_state.cpp:228-244) and the logical cache."""
    kv = []
    for j in range(g.n_qsa + 1):
        index = j < g.n_qsa
        lay = O.kv_layout(0, tokens, index, g)
        kv.append({"format": 0, "cells": lay["cells"], "heads": g.n_head_kv, "head_dim": g.head_dim, "page_size": 4,
                   "pooled_rows": lay["pooled_rows"], "idx_dim": g.idx_key_dim,
                   "k": s.k[j][:lay["data"]].tobytes(), "v": s.v[j][:lay["value_data"]].tobytes(),
                   "k_scale": b"", "v_scale": b"",
                   "pooled": s.pooled[j].view(np.uint8)[:lay["pooled"]].tobytes() if index else b""})
    live = {"ids": s.ids, "imgs": [], "gdn": s.gdn.tobytes(), "ple": b"" if s.ple is None else s.ple.tobytes(),
            "tails": b"".join(t.tobytes() for t in s.tail), "dead": b"".join(d.tobytes() for d in s.dead),
            "block_pos": b"".join(b.tobytes() for b in s.block_pos), "used": 0, "stage_parts": []}
    return {"geometry": g.key(), "layer_lo": 0, "layer_hi": g.n_layers, "cvec": True, "kv": kv, "live": live,
            "checkpoints": [], "stage_parts": []}


def test_fnv_matches_golden_payload_hash():
    for t, rec in G["small"].items():
        data = payload(t)
        assert len(data) == rec["bytes"]
        assert O.fnv1a64(data) == rec["payload_hash"]


@pytest.mark.parametrize("t", [1, 5, 257])
def test_oracle_encodes_the_golden_payload(t):
    """The oracle's cache + layout + encoder reproduce the reference's payload byte for byte."""
    s = O.make_sequence(SMALL, t, seed=7)
    img = oracle_image(SMALL, s, t)
    p = sr4h.Payload(payload(t))
    assert sr4h.encode(img, p.geom_hash, p.pack_hash) == payload(t)


@pytest.mark.parametrize("t", [1, 5, 257])
def test_gather_from_permuted_pool_equals_golden_blobs(t):
    """The block-table rule: scatter the logical cache into a permuted pool, gather it back through the
    table, and the bytes are exactly the K/V blobs the reference saved from its identity pool."""
    s = O.make_sequence(SMALL, t, seed=7)
    p = sr4h.Payload(payload(t))
    pb = SMALL.page_bytes
    pages = O.pages_for(t)
    for j in range(SMALL.n_qsa + 1):
        table = O.permutation(pages * 3, seed=100 + j)[:pages]
        pool = np.zeros(pages * 3 * pb, dtype=np.uint8)
        O.scatter_pages(s.k[j], table, pages, pb, pool)
        assert O.gather_pages(pool, table, pages, pb).tobytes() == bytes(p.blob(p.kv[j]["k"]))


def test_layout_matches_reference_records():
    for t in (1, 5, 257):
        p = sr4h.Payload(payload(t))
        for j, kv in enumerate(p.kv):
            lay = O.kv_layout(0, t, j < SMALL.n_qsa, SMALL)
            assert (kv["cells"], kv["pooled_rows"], kv["k"][0], kv["v"][0], kv["pooled"][0]) == \
                (lay["cells"], lay["pooled_rows"], lay["data"], lay["value_data"], lay["pooled"])
        z = O.state_sizes(SMALL)
        assert p.live["gdn"][0] == z["gdn"]
        assert p.live["tails"][0] == SMALL.n_qsa * z["tail"]


def test_layout_quantized_formats():
    g = O.Geometry()
    # int8: 1 byte per value + fp16 scale per 64; q4_0: 144 B per cell and head at head_dim 256; hybrid K8V4
    assert O.kv_layout(1, 5, True, g)["scales"] == 8 * 2 * 4 * 2
    assert O.kv_layout(2, 5, True, g)["data"] == 8 * 2 * 144
    h = O.kv_layout(3, 5, True, g)
    assert h["data"] == 8 * 2 * 256 and h["value_data"] == 8 * 2 * 144 and h["value_scales"] == 0
    assert O.kv_layout(0, -1, True, g) is None


@pytest.mark.slow
def test_config1_blob_hashes():
    """Config 1 at full geometry: every blob the reference saved, re-derived from the oracle."""
    c = G["config1"]
    g = O.Geometry()
    s = O.make_sequence(g, c["tokens"], seed=c["seed"])
    pages = O.pages_for(c["tokens"])
    for j, rec in enumerate(c["blobs"]["kv"]):
        assert rec["k"] == [pages * g.page_bytes, O.fnv1a64(s.k[j])]
        assert rec["v"] == [pages * g.page_bytes, O.fnv1a64(s.v[j])]
    assert c["blobs"]["live"]["gdn"] == [g.gdn_bytes, O.fnv1a64(s.gdn)]
    assert c["blobs"]["live"]["ids"] == O.fnv1a64(s.ids.tobytes())
    assert O.metric_bytes(g, c["tokens"]) == 179716096


@pytest.mark.slow
def test_config2a_32k_blob_hashes():
    """Config 2(a)'s length at full geometry (32,768 tokens, seed 2): the K/V of every layer, the GDN rows and the
    ids the reference saved, re-derived from the oracle.  The GPU test of the full-size pool->pool hand-off checks
    its destination against the same reference-written hashes."""
    c = G["config2a_32k"]
    g = O.Geometry()
    s = O.make_sequence(g, c["tokens"], seed=c["seed"])
    pages = O.pages_for(c["tokens"])
    assert len(c["blobs"]["kv"]) == g.n_qsa + 1
    for j, rec in enumerate(c["blobs"]["kv"]):
        assert rec["k"] == [pages * g.page_bytes, O.fnv1a64(s.k[j])]
        assert rec["v"] == [pages * g.page_bytes, O.fnv1a64(s.v[j])]
    assert c["blobs"]["live"]["gdn"] == [g.gdn_bytes, O.fnv1a64(s.gdn)]
    assert c["blobs"]["live"]["ids"] == O.fnv1a64(s.ids.tobytes())
    assert O.metric_bytes(g, c["tokens"]) == 884_473_856


def test_f16_rounding_is_nearest_even():
    lib = O.lib()
    assert lib.orc_f32_to_f16(1.0) == 0x3C00
    assert lib.orc_f32_to_f16(65504.0) == 0x7BFF
    assert lib.orc_f32_to_f16(65520.0) == 0x7C00        # rounds up to inf
    assert lib.orc_f32_to_f16(1.0 + 2.0 ** -11) == 0x3C00  # tie -> even
    assert lib.orc_f32_to_f16(1.0 + 3 * 2.0 ** -11) == 0x3C02
    assert lib.orc_f32_to_f16(2.0 ** -24) == 0x0001      # smallest subnormal
    x = np.array([0.1, -2.5, 3.14159, 1e-6, 7e4], dtype=np.float32)
    assert [lib.orc_f32_to_f16(float(v)) for v in x] == list(x.astype(np.float16).view(np.uint16))


def test_generators_are_counter_based():
    a = O.f16_normal(1000, seed=3)
    b = O.f16_normal(500, seed=3, offset=500)
    assert (a[500:] == b).all()
    v = O.f32_normal(200000, seed=5, sigma=0.02)
    assert abs(v.mean()) < 1e-3 and abs(v.std() - 0.02) < 1e-3
    p = O.permutation(1000, seed=9)
    assert sorted(p.tolist()) == list(range(1000))


@needs_ref
@pytest.mark.parametrize("t", [2, 4, 63, 64, 255, 256, 1024])
def test_live_reference_agrees_with_oracle(t):
    """Fresh shapes and seeds against the live reference: save+encode equals the oracle's encoding."""
    s = O.make_sequence(SMALL, t, seed=t + 11)
    data, h = O.ref_snapshot_encode(O.RefPools(s), s.ids, 5, 6)
    assert sr4h.encode(oracle_image(SMALL, s, t), 5, 6) == data
    assert O.fnv1a64(data) == h


@needs_ref
def test_live_reference_round_trip_and_refusals():
    t = 257
    s = O.make_sequence(SMALL, t, seed=3, with_ple=True)
    data, _ = O.ref_snapshot_encode(O.RefPools(s), s.ids)
    dst = O.RefPools(s, empty=True)
    rc, msg = O.ref_decode_restore(dst, data)
    assert rc == 0, msg
    n = O.kv_layout(0, t, True, SMALL)["data"]
    for j in range(SMALL.n_qsa + 1):
        assert (dst.k[j][:n] == s.k[j][:n]).all() and (dst.v[j][:n] == s.v[j][:n]).all()
    assert (dst.gdn == s.gdn).all() and (dst.ple == s.ple).all()
    # a corrupted payload is refused by the decoder and leaves the pools untouched
    bad = bytearray(data)
    bad[0] ^= 1
    fresh = O.RefPools(s, empty=True)
    rc, msg = O.ref_decode_restore(fresh, bytes(bad))
    assert rc == 4 and all((a == 0).all() for a in fresh.k)
    # an empty conversation is refused by the reference's own validation
    with pytest.raises(RuntimeError, match="invalid live token"):
        O.ref_snapshot_encode(O.RefPools(s), np.zeros(0, dtype=np.int32))


@needs_ref
def test_live_reference_transfer_failure_is_reported():
    """Host-side fault injection, the reference's own way (the Nth wrapped copy fails)."""
    t = 64
    s = O.make_sequence(SMALL, t, seed=4)
    data, _ = O.ref_snapshot_encode(O.RefPools(s), s.ids)
    O.ref().ref_fail_copy_at(3)
    try:
        rc, msg = O.ref_decode_restore(O.RefPools(s, empty=True), data)
    finally:
        O.ref().ref_fail_copy_at(0)
    assert rc == 6 and "copy" in msg


@needs_ref
def test_live_reference_wire_timing_round_trips():
    """The timing hook the CPU sweep uses: the reference's encode then decode (hash-checked) of a payload."""
    s = O.make_sequence(SMALL, 100, seed=8)
    data, _ = O.ref_snapshot_encode(O.RefPools(s), s.ids)
    enc, dec = O.ref_time_wire(data, 3)
    assert len(enc) == len(dec) == 3 and (enc > 0).all() and (dec > 0).all()
