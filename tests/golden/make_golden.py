"""Generate the golden fixtures in tests/golden/ from the REFERENCE's own code (oracle/_ref/libstrata_ref.so).

    make -C oracle && python tests/golden/make_golden.py

Outputs
  ref_payload_T{T}.bin   SR4H payloads written by the reference's conversation_snapshot_save +
                         conversation_wire_encode for a small geometry (SMALL below), seed 7.
  golden.json            for each small payload: its FNV-1a payload hash; for config 1 (the full geometry,
                         4,096 tokens, seed 1) and for config 2(a)'s length (32,768 tokens, seed 2): the
                         payload size and hash plus the FNV-1a of every blob the reference wrote (per-layer K
                         and V, pooled rows, the running state, the ids).

The synthetic inputs come from oracle/kv_oracle.c's seeded generators, so any machine regenerates the same
caches; the fixtures pin what the reference makes of them.
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402
import sr4h  # noqa: E402

SMALL = dict(n_layers=8, qsa_interval=4, n_head_kv=2, head_dim=64, ssm_state_size=4, ssm_v_heads=2,
             ssm_conv_channels=16, idx_key_dim=8)
SMALL_TOKENS = [1, 5, 257]
CONFIG1_TOKENS = 4096
CONFIG2A_TOKENS, CONFIG2A_SEED = 32768, 2
GEOM_HASH, PACK_HASH = 0x1111222233334444, 0x5555666677778888


def blob_hashes(p: sr4h.Payload) -> dict:
    out = {"kv": []}
    for kv in p.kv:
        out["kv"].append({n: [kv[n][0], O.fnv1a64(p.blob(kv[n]))] for n in sr4h.KV_BUFFERS})
    out["live"] = {n: [p.live[n][0], O.fnv1a64(p.blob(p.live[n]))] for n in sr4h.CP_BUFFERS}
    out["live"]["ids"] = O.fnv1a64(p.live["ids"].tobytes())
    return out


def main() -> None:
    if not O.ref_available():
        sys.exit("oracle/_ref/libstrata_ref.so is not built (needs the reference tree): make -C oracle ref")
    golden = {"small_geometry": SMALL, "small": {}, "config1": {}}
    g = O.Geometry(**SMALL)
    for t in SMALL_TOKENS:
        s = O.make_sequence(g, t, seed=7)
        data, h = O.ref_snapshot_encode(O.RefPools(s), s.ids, GEOM_HASH, PACK_HASH)
        with open(os.path.join(HERE, f"ref_payload_T{t}.bin"), "wb") as f:
            f.write(data)
        golden["small"][str(t)] = {"bytes": len(data), "payload_hash": h}
    g = O.Geometry()
    s = O.make_sequence(g, CONFIG1_TOKENS, seed=1)
    data, h = O.ref_snapshot_encode(O.RefPools(s), s.ids, GEOM_HASH, PACK_HASH)
    p = sr4h.Payload(data)
    golden["config1"] = {"tokens": CONFIG1_TOKENS, "seed": 1, "bytes": len(data), "payload_hash": h,
                         "snapshot_bytes": O.ref_snapshot_bytes(O.RefPools(s), s.ids), "blobs": blob_hashes(p)}
    s = O.make_sequence(g, CONFIG2A_TOKENS, seed=CONFIG2A_SEED)
    data, h = O.ref_snapshot_encode(O.RefPools(s), s.ids, GEOM_HASH, PACK_HASH)
    golden["config2a_32k"] = {"tokens": CONFIG2A_TOKENS, "seed": CONFIG2A_SEED, "bytes": len(data), "payload_hash": h,
                              "blobs": blob_hashes(sr4h.Payload(data))}
    del s, data
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(golden, f, indent=1, sort_keys=True)
    print("wrote", len(SMALL_TOKENS), "payloads and golden.json")


if __name__ == "__main__":
    main()
