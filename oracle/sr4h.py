"""oracle/sr4h.py - TEST INFRASTRUCTURE: the SR4H hand-off payload format, restated in Python.

The checker for the wire codec and for parsing the reference's own payloads into comparable blobs.  Never
the product.  The format is the reference's (include/strata/core/conversation_wire.hpp:24-81; the emitter
order in src/core/conversation_wire.cpp:260-470):

    payload := header_record(256) body_records zero_pad(to 64) blob_pool
    records := KV[n_kv] CHECKPOINT(live) CHECKPOINT[n_checkpoints] STAGE[n_stage_parts] END!
    record  := {u32 kind; u32 flags=0; u64 bytes} body
    BLOBREF := {u64 bytes; u64 offset-from-payload-start}; zero-length buffers are {0,0} with no pool entry
    pool entries start on 64-byte boundaries (pool-relative), gaps zero-filled, the pool rounded up to 64.

An image is a plain dict:
    {"geometry": [18 ints], "layer_lo", "layer_hi", "cvec": bool,
     "kv": [KV...], "live": CP, "checkpoints": [CP...], "stage_parts": [{"layer_lo","layer_hi","state": CP, "kv": [KV...]}]}
    KV = {"format","cells","heads","head_dim","page_size","pooled_rows","idx_dim",
          "k","v","k_scale","v_scale","pooled"}              (buffers are bytes-like)
    CP = {"ids": int32 array, "imgs": [(start, hash)], "gdn","ple","tails","dead","block_pos": bytes-like,
          "used": int, "stage_parts": [CP...]}
"""
from __future__ import annotations

import struct

import numpy as np

MAGIC = 0x48345253          # 'S','R','4','H' little-endian
VERSION = 1
HEADER_BYTES = 256
RECORD_HEADER_BYTES = 16
BLOB_ALIGN = 64
KIND_KV, KIND_CHECKPOINT, KIND_STAGE, KIND_END = 1, 2, 3, 0x21444E45
FLAG_CVEC, FLAG_STAGE_PARTS, FLAG_PARTIAL = 1, 2, 4
KV_BODY_BYTES = 136
KV_BUFFERS = ("k", "v", "k_scale", "v_scale", "pooled")
CP_BUFFERS = ("gdn", "ple", "tails", "dead", "block_pos")
FNV_SEED = 1469598103934665603


def round_up_64(n: int) -> int:
    return (n + 63) & ~63


def _nbytes(b) -> int:
    return 0 if b is None else memoryview(b).nbytes


class _Writer:
    """Two-pass emitter: pass 1 assigns pool offsets (emission order), pass 2 writes the same traversal."""

    def __init__(self, image: dict):
        self.image = image
        self.blobs: list = []          # (buffer, pool-relative offset)
        self.pool_rel = 0
        self.pool_off = 0
        self.layout = True
        self.index = 0
        self.out = bytearray()

    def blob(self, buf) -> int:
        n = _nbytes(buf)
        if n == 0:
            return 0
        if self.layout:
            rel = round_up_64(self.pool_rel)
            self.pool_rel = rel + n
            self.blobs.append((buf, rel))
            return 0
        rel = self.blobs[self.index][1]
        self.index += 1
        return self.pool_off + rel

    def kv_record(self, kv: dict) -> None:
        self.out += struct.pack("<IIQ", KIND_KV, 0, KV_BODY_BYTES)
        self.out += struct.pack("<iI6q", kv["format"], 0, kv["cells"], kv["heads"], kv["head_dim"], kv["page_size"],
                                kv["pooled_rows"], kv["idx_dim"])
        for name in KV_BUFFERS:
            buf = kv.get(name)
            off = self.blob(buf)
            self.out += struct.pack("<QQ", _nbytes(buf), off)

    @staticmethod
    def checkpoint_body_bytes(cp: dict) -> int:
        n_ids = len(cp["ids"])
        n = 8 + 4 * n_ids + (4 if (n_ids * 4) % 8 else 0)
        n += 8 + 16 * len(cp.get("imgs", []))
        n += 5 * 16 + 8 + 8
        for part in cp.get("stage_parts", []):
            n += RECORD_HEADER_BYTES + _Writer.checkpoint_body_bytes(part)
        return n

    def checkpoint_record(self, cp: dict) -> None:
        self.out += struct.pack("<IIQ", KIND_CHECKPOINT, 0, self.checkpoint_body_bytes(cp))
        ids = np.ascontiguousarray(cp["ids"], dtype="<i4")
        self.out += struct.pack("<Q", len(ids)) + ids.tobytes()
        if (len(ids) * 4) % 8:
            self.out += b"\0" * 4
        imgs = cp.get("imgs", [])
        self.out += struct.pack("<Q", len(imgs))
        for start, h in imgs:
            self.out += struct.pack("<qQ", start, h)
        for name in CP_BUFFERS:
            buf = cp.get(name)
            off = self.blob(buf)
            self.out += struct.pack("<QQ", _nbytes(buf), off)
        parts = cp.get("stage_parts", [])
        self.out += struct.pack("<QQ", cp.get("used", 0), len(parts))
        for part in parts:
            self.checkpoint_record(part)

    def stage_record(self, st: dict) -> None:
        body = 16 + RECORD_HEADER_BYTES + self.checkpoint_body_bytes(st["state"]) + 8 + \
            len(st["kv"]) * (RECORD_HEADER_BYTES + KV_BODY_BYTES)
        self.out += struct.pack("<IIQ", KIND_STAGE, 0, body)
        self.out += struct.pack("<qq", st["layer_lo"], st["layer_hi"])
        self.checkpoint_record(st["state"])
        self.out += struct.pack("<Q", len(st["kv"]))
        for kv in st["kv"]:
            self.kv_record(kv)

    def body(self) -> None:
        img = self.image
        for kv in img["kv"]:
            self.kv_record(kv)
        self.checkpoint_record(img["live"])
        for cp in img.get("checkpoints", []):
            self.checkpoint_record(cp)
        for st in img.get("stage_parts", []):
            self.stage_record(st)
        self.out += struct.pack("<IIQ", KIND_END, 0, 0)


def encode(image: dict, geom_hash: int = 0, pack_hash: int = 0) -> bytes:
    """The payload bytes of `image` (the reference's conversation_wire_encode output)."""
    w = _Writer(image)
    w.body()                                   # pass 1: body size and pool offsets
    body_bytes = len(w.out)
    w.pool_off = round_up_64(HEADER_BYTES + body_bytes)
    pool_bytes = round_up_64(w.pool_rel) if w.blobs else 0
    total = w.pool_off + pool_bytes
    flags = (FLAG_CVEC if image.get("cvec", True) else 0) | (FLAG_STAGE_PARTS if image.get("stage_parts") else 0)
    header = struct.pack("<IHH18Q", MAGIC, VERSION, flags, *[g & (2**64 - 1) for g in image["geometry"]])
    header += struct.pack("<QQqqqqQQQQQQQ", image["layer_lo"], image["layer_hi"], len(image["kv"]),
                          len(image.get("checkpoints", [])), len(image.get("stage_parts", [])),
                          len(image["live"]["ids"]), w.pool_off, pool_bytes, geom_hash, pack_hash, total, 0, 0)
    assert len(header) == HEADER_BYTES
    w.layout = False
    w.index = 0
    w.out = bytearray()
    w.body()                                   # pass 2: the same traversal, real offsets
    out = bytearray(total)
    out[:HEADER_BYTES] = header
    out[HEADER_BYTES:HEADER_BYTES + len(w.out)] = w.out
    for buf, rel in w.blobs:
        mv = memoryview(buf).cast("B")
        out[w.pool_off + rel:w.pool_off + rel + mv.nbytes] = mv
    return bytes(out)


# ------------------------------------------------------------------------------------------------ parse

class Payload:
    """A parsed payload: the header fields and the records, with blobs as (bytes, offset) references."""

    def __init__(self, data):
        self.data = memoryview(data).cast("B")
        h = struct.unpack_from("<IHH18Q", self.data, 0)
        if h[0] != MAGIC or h[1] != VERSION:
            raise ValueError("not an SR4H v1 payload")
        self.flags = h[2]
        self.geometry = [struct.unpack("<q", struct.pack("<Q", g))[0] for g in h[3:21]]
        (self.layer_lo, self.layer_hi, self.n_kv, self.n_checkpoints, self.n_stage_parts, self.live_tokens,
         self.blob_pool_off, self.blob_pool_bytes, self.geom_hash, self.pack_hash, self.payload_bytes,
         self.payload_hash_field, self.reserved) = struct.unpack_from("<QQqqqqQQQQQQQ", self.data, 152)
        self.pos = HEADER_BYTES
        self.kv = [self._kv() for _ in range(self.n_kv)]
        self.live = self._checkpoint()
        self.checkpoints = [self._checkpoint() for _ in range(self.n_checkpoints)]
        self.stage_parts = [self._stage() for _ in range(self.n_stage_parts)]
        kind, flags, n = struct.unpack_from("<IIQ", self.data, self.pos)
        if kind != KIND_END or flags or n:
            raise ValueError("missing END! record")
        self.pos += RECORD_HEADER_BYTES

    def blob(self, ref) -> memoryview:
        n, off = ref
        return self.data[off:off + n] if n else self.data[0:0]

    def _record(self, want: int) -> int:
        kind, flags, n = struct.unpack_from("<IIQ", self.data, self.pos)
        if kind != want or flags:
            raise ValueError(f"expected record kind {want}, found {kind:#x}")
        self.pos += RECORD_HEADER_BYTES
        return n

    def _kv(self) -> dict:
        self._record(KIND_KV)
        f = struct.unpack_from("<iI6q", self.data, self.pos)
        self.pos += 56
        refs = [struct.unpack_from("<QQ", self.data, self.pos + 16 * i) for i in range(5)]
        self.pos += 80
        kv = dict(zip(("format", "pad", "cells", "heads", "head_dim", "page_size", "pooled_rows", "idx_dim"), f))
        for name, ref in zip(KV_BUFFERS, refs):
            kv[name] = ref
        return kv

    def _checkpoint(self) -> dict:
        self._record(KIND_CHECKPOINT)
        (n_ids,) = struct.unpack_from("<Q", self.data, self.pos)
        self.pos += 8
        ids = np.frombuffer(self.data, dtype="<i4", count=n_ids, offset=self.pos).copy()
        self.pos += 4 * n_ids + (4 if (n_ids * 4) % 8 else 0)
        (n_imgs,) = struct.unpack_from("<Q", self.data, self.pos)
        self.pos += 8
        imgs = [struct.unpack_from("<qQ", self.data, self.pos + 16 * i) for i in range(n_imgs)]
        self.pos += 16 * n_imgs
        cp = {"ids": ids, "imgs": imgs}
        for i, name in enumerate(CP_BUFFERS):
            cp[name] = struct.unpack_from("<QQ", self.data, self.pos + 16 * i)
        self.pos += 80
        cp["used"], n_parts = struct.unpack_from("<QQ", self.data, self.pos)
        self.pos += 16
        cp["stage_parts"] = [self._checkpoint() for _ in range(n_parts)]
        return cp

    def _stage(self) -> dict:
        self._record(KIND_STAGE)
        lo, hi = struct.unpack_from("<qq", self.data, self.pos)
        self.pos += 16
        state = self._checkpoint()
        (n_kv,) = struct.unpack_from("<Q", self.data, self.pos)
        self.pos += 8
        return {"layer_lo": lo, "layer_hi": hi, "state": state, "kv": [self._kv() for _ in range(n_kv)]}

    def materialize(self) -> dict:
        """The payload as an encode()-able image dict (blobs copied out as bytes)."""
        def kv(k):
            d = {n: k[n] for n in ("format", "cells", "heads", "head_dim", "page_size", "pooled_rows", "idx_dim")}
            for name in KV_BUFFERS:
                d[name] = bytes(self.blob(k[name]))
            return d

        def cp(c):
            d = {"ids": c["ids"], "imgs": c["imgs"], "used": c["used"], "stage_parts": [cp(p) for p in c["stage_parts"]]}
            for name in CP_BUFFERS:
                d[name] = bytes(self.blob(c[name]))
            return d

        return {"geometry": self.geometry, "layer_lo": self.layer_lo, "layer_hi": self.layer_hi,
                "cvec": bool(self.flags & FLAG_CVEC), "kv": [kv(k) for k in self.kv], "live": cp(self.live),
                "checkpoints": [cp(c) for c in self.checkpoints],
                "stage_parts": [{"layer_lo": s["layer_lo"], "layer_hi": s["layer_hi"], "state": cp(s["state"]),
                                 "kv": [kv(k) for k in s["kv"]]} for s in self.stage_parts]}
