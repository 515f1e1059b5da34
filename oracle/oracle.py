"""oracle/oracle.py - TEST INFRASTRUCTURE: Python access to the CPU checkers.

  * liboracle.so          the C restatement (kv_oracle.c): seeded inputs, block-table gather/scatter,
                          snapshot extents, FNV-1a.
  * _ref/libstrata_ref.so the reference's own park/resume + codec sources, compiled by oracle/Makefile
                          (present wherever `make -C oracle` ran with the reference tree available).

Only tests/, tests/golden/make_golden.py, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.  The product never does.
"""
from __future__ import annotations

import ctypes as C
import math
import os
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libstrata_ref.so")

PAGE_CELLS = 4          # include/strata/kernels/qsa.hpp:115
IDX_BLOCK = 4           # include/strata/kernels/qsa.hpp:112
BLOCK_TOKENS = 256      # the configs' block granule
PLE_BYTES = 9 * 10240 * 4
FNV_SEED = 1469598103934665603


@dataclass
class Geometry:
    """The ModelGeometry fields this path reads (include/strata/core/layout.hpp:27-60), at the configs' values."""
    n_layers: int = 48
    qsa_interval: int = 4
    n_head_kv: int = 2
    head_dim: int = 256
    ssm_state_size: int = 128
    ssm_v_heads: int = 32
    ssm_d_conv: int = 4
    ssm_conv_channels: int = 8192
    idx_key_dim: int = 128

    @property
    def n_qsa(self) -> int:
        return self.n_layers // self.qsa_interval

    @property
    def n_gdn(self) -> int:
        return self.n_layers - self.n_qsa

    @property
    def page_bytes(self) -> int:
        return self.n_head_kv * PAGE_CELLS * self.head_dim * 2

    @property
    def gdn_row_floats(self) -> int:
        s = self.ssm_state_size
        return s * self.ssm_v_heads * s + self.ssm_conv_channels * (self.ssm_d_conv - 1)

    @property
    def gdn_bytes(self) -> int:
        return self.n_gdn * self.gdn_row_floats * 4

    def key(self) -> list:
        """geometry_key(g) (src/core/conversation_state.cpp:14-19) with ModelGeometry's other defaults."""
        return [2560, self.n_layers, self.qsa_interval, self.ssm_state_size, 16, self.ssm_v_heads, self.ssm_d_conv,
                self.ssm_conv_channels, 6144, 24, self.n_head_kv, self.head_dim, 4, self.idx_key_dim, 4, 320, 512, 640]


def pages_for(tokens: int) -> int:
    return (tokens + PAGE_CELLS - 1) // PAGE_CELLS


def metric_bytes(g: Geometry, tokens: int) -> int:
    """B(T): K+V of every QSA layer over ceil(T/4) pages, the GDN rows, the token ids."""
    return 2 * g.n_qsa * pages_for(tokens) * g.page_bytes + g.gdn_bytes + 4 * tokens


# ------------------------------------------------------------------------------------------------ liboracle

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_LIB):
            raise RuntimeError(f"{ORACLE_LIB} is not built: run `make -C oracle`")
        L = C.CDLL(ORACLE_LIB)
        P = C.c_void_p
        u64, i64, i32 = C.c_uint64, C.c_int64, C.c_int32
        L.orc_fill_f16_normal.argtypes = [P, u64, u64, u64]
        L.orc_fill_f32_normal.argtypes = [P, u64, u64, u64, C.c_float]
        L.orc_fill_ids.argtypes = [P, u64, u64, i32]
        L.orc_permutation.argtypes = [P, i64, u64]
        L.orc_f32_to_f16.argtypes = [C.c_float]
        L.orc_f32_to_f16.restype = C.c_uint16
        L.orc_expand_block_table.argtypes = [P, i64, i64, i64, i64, P]
        L.orc_gather_pages.argtypes = [P, P, i64, u64, P]
        L.orc_scatter_pages.argtypes = [P, P, i64, u64, P]
        L.orc_kv_layout.argtypes = [C.c_int32, i64, C.c_int, i64, i64, i64, P]
        L.orc_state_sizes.argtypes = [i64, i64, i64, i64, i64, i64, i64, P]
        L.orc_fnv1a64.argtypes = [P, u64, u64]
        L.orc_fnv1a64.restype = u64
        L.orc_page_checksum.argtypes = [P, i64, u64]
        L.orc_page_checksum.restype = u64
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def f16_normal(n: int, seed: int, offset: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    lib().orc_fill_f16_normal(_p(out), n, seed, offset)
    return out


def f32_normal(n: int, seed: int, sigma: float, offset: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().orc_fill_f32_normal(_p(out), n, seed, offset, sigma)
    return out


def token_ids(n: int, seed: int, vocab: int = 151936) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    lib().orc_fill_ids(_p(out), n, seed, vocab)
    return out


def permutation(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    lib().orc_permutation(_p(out), n, seed)
    return out


def expand_block_table(blocks: np.ndarray, pages_per_block: int, slot_pages: int, page_offset: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.int32)
    out = np.empty(len(blocks) * pages_per_block, dtype=np.int32)
    lib().orc_expand_block_table(_p(blocks), len(blocks), pages_per_block, slot_pages, page_offset, _p(out))
    return out


def gather_pages(pool: np.ndarray, table: np.ndarray, n_pages: int, page_bytes: int) -> np.ndarray:
    table = np.ascontiguousarray(table, dtype=np.int32)
    assert len(table) >= n_pages and pool.dtype == np.uint8
    assert n_pages == 0 or int(table[:n_pages].max()) * page_bytes + page_bytes <= pool.nbytes
    out = np.empty(n_pages * page_bytes, dtype=np.uint8)
    lib().orc_gather_pages(_p(pool), _p(table), n_pages, page_bytes, _p(out))
    return out


def scatter_pages(image: np.ndarray, table: np.ndarray, n_pages: int, page_bytes: int, pool: np.ndarray) -> None:
    table = np.ascontiguousarray(table, dtype=np.int32)
    assert image.nbytes >= n_pages * page_bytes and pool.dtype == np.uint8
    assert n_pages == 0 or int(table[:n_pages].max()) * page_bytes + page_bytes <= pool.nbytes
    lib().orc_scatter_pages(_p(image), _p(table), n_pages, page_bytes, _p(pool))


class _KvLayout(C.Structure):
    _fields_ = [("format", C.c_int32), ("cells", C.c_int64), ("pooled_rows", C.c_int64), ("data", C.c_uint64),
                ("scales", C.c_uint64), ("pooled", C.c_uint64), ("value_data", C.c_uint64),
                ("value_scales", C.c_uint64)]


def kv_layout(fmt: int, upto: int, index: bool, g: Geometry) -> dict | None:
    out = _KvLayout()
    if lib().orc_kv_layout(fmt, upto, int(index), g.n_head_kv, g.head_dim, g.idx_key_dim, C.byref(out)):
        return None
    return {f: getattr(out, f) for f, _ in _KvLayout._fields_}


class _StateSizes(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("gdn", "ple", "tail", "dead", "block_pos")]


def state_sizes(g: Geometry) -> dict:
    out = _StateSizes()
    rc = lib().orc_state_sizes(g.n_layers, g.qsa_interval, g.ssm_state_size, g.ssm_v_heads, g.ssm_d_conv,
                               g.ssm_conv_channels, g.idx_key_dim, C.byref(out))
    assert rc == 0
    return {f: getattr(out, f) for f, _ in _StateSizes._fields_}


def fnv1a64(data, seed: int = FNV_SEED) -> int:
    a = np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8)
    return int(lib().orc_fnv1a64(a.ctypes.data, a.nbytes, seed))


def page_checksum(data, page_bytes: int) -> int:
    a = np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8)
    assert a.nbytes % page_bytes == 0
    return int(lib().orc_page_checksum(a.ctypes.data, a.nbytes // page_bytes, page_bytes))


# ------------------------------------------------------------------------------------------------ synthetic caches

@dataclass
class Sequence:
    """One sequence's cache in LOGICAL order (what the reference's identity-layout pools hold)."""
    g: Geometry
    tokens: int
    seed: int
    k: list = field(default_factory=list)        # per QSA layer (+ draft last), uint8 images of pages*page_bytes
    v: list = field(default_factory=list)
    pooled: list = field(default_factory=list)   # per QSA layer, float32 (pooled_capacity_rows, idx_dim)
    tail: list = field(default_factory=list)
    dead: list = field(default_factory=list)
    block_pos: list = field(default_factory=list)
    gdn: np.ndarray | None = None
    ple: np.ndarray | None = None
    ids: np.ndarray | None = None

    @property
    def pages(self) -> int:
        return pages_for(self.tokens)

    @property
    def pooled_capacity_rows(self) -> int:
        return self.pages * PAGE_CELLS // IDX_BLOCK + 2


def layer_seed(seed: int, layer: int, which: int) -> int:
    return (seed * 1000003 + layer * 7919 + which * 104729) & 0xFFFFFFFFFFFFFFFF


def make_sequence(g: Geometry, tokens: int, seed: int, with_ple: bool = False) -> Sequence:
    """The configs' synthetic cache: K/V fp16 ~N(0,1), GDN/conv state fp32 ~N(0,0.02), ids uniform; the draft
    layer (index n_qsa) and the indexer buffers too, because the reference saves them on every park."""
    s = Sequence(g, tokens, seed)
    n16 = s.pages * g.page_bytes // 2
    for layer in range(g.n_qsa + 1):
        s.k.append(f16_normal(n16, layer_seed(seed, layer, 1)).view(np.uint8))
        s.v.append(f16_normal(n16, layer_seed(seed, layer, 2)).view(np.uint8))
    for layer in range(g.n_qsa):
        s.pooled.append(f32_normal(s.pooled_capacity_rows * g.idx_key_dim, layer_seed(seed, layer, 3), 1.0))
        s.tail.append(f32_normal((IDX_BLOCK - 1) * g.idx_key_dim, layer_seed(seed, layer, 4), 1.0))
        s.dead.append(f32_normal(g.idx_key_dim, layer_seed(seed, layer, 5), 1.0))
        s.block_pos.append(np.array([tokens // IDX_BLOCK], dtype=np.int32))
    s.gdn = f32_normal(g.n_gdn * g.gdn_row_floats, layer_seed(seed, 999, 6), 0.02)
    s.ple = f32_normal(PLE_BYTES // 4, layer_seed(seed, 999, 7), 1.0) if with_ple else None
    s.ids = token_ids(tokens, layer_seed(seed, 999, 8))
    return s


# ------------------------------------------------------------------------------------------------ the reference

MAX_QSA = 64


class RefSession(C.Structure):
    _fields_ = [(n, C.c_int64) for n in ("n_layers", "qsa_interval", "n_head_kv", "head_dim", "ssm_state_size",
                                         "ssm_v_heads", "ssm_d_conv", "ssm_conv_channels", "idx_key_dim",
                                         "max_cells", "idx_pooled_rows")] + [
        ("k_pool", C.c_void_p * (MAX_QSA + 1)), ("v_pool", C.c_void_p * (MAX_QSA + 1)),
        ("idx_pooled", C.c_void_p * MAX_QSA), ("idx_tail", C.c_void_p * MAX_QSA),
        ("idx_dead", C.c_void_p * MAX_QSA), ("idx_block_pos", C.c_void_p * MAX_QSA),
        ("gdn_state", C.c_void_p), ("ple_hist", C.c_void_p)]


_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def ref() -> C.CDLL:
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError(f"{REF_LIB} is not built (needs the reference tree): run `make -C oracle ref`")
        L = C.CDLL(REF_LIB)
        P, u64, i64 = C.c_void_p, C.c_uint64, C.c_int64
        L.ref_snapshot_encode.argtypes = [P, i64, P, u64, u64, C.POINTER(P), C.POINTER(u64), C.POINTER(u64), C.c_char_p,
                                          C.c_size_t]
        L.ref_decode_restore.argtypes = [P, P, u64, C.c_char_p, C.c_size_t]
        L.ref_snapshot_bytes.argtypes = [P, i64, P, C.POINTER(u64), C.c_char_p, C.c_size_t]
        L.ref_time_park_resume.argtypes = [P, P, i64, P, C.c_int, P, P, C.c_char_p, C.c_size_t]
        L.ref_time_wire.argtypes = [P, u64, C.c_int, P, P, C.c_char_p, C.c_size_t]
        L.ref_payload_hash.argtypes = [P, u64]
        L.ref_payload_hash.restype = u64
        L.ref_fail_copy_at.argtypes = [C.c_int]
        L.ref_free.argtypes = [P]
        _ref = L
    return _ref


class RefPools:
    """Identity-layout host pools holding a Sequence, bound into a RefSession (the arrays stay alive here)."""

    def __init__(self, seq: Sequence, empty: bool = False):
        g = seq.g
        self.seq = seq
        self.arrays = []
        r = RefSession()
        for name in ("n_layers", "qsa_interval", "n_head_kv", "head_dim", "ssm_state_size", "ssm_v_heads",
                     "ssm_d_conv", "ssm_conv_channels", "idx_key_dim"):
            setattr(r, name, getattr(g, name))
        r.max_cells = seq.pages * PAGE_CELLS
        r.idx_pooled_rows = seq.pooled_capacity_rows

        def keep(a):
            a = np.zeros_like(a) if empty else np.array(a, copy=True)
            self.arrays.append(a)
            return a

        self.k = [keep(a) for a in seq.k]
        self.v = [keep(a) for a in seq.v]
        self.pooled = [keep(a) for a in seq.pooled]
        self.tail = [keep(a) for a in seq.tail]
        self.dead = [keep(a) for a in seq.dead]
        self.block_pos = [keep(a) for a in seq.block_pos]
        self.gdn = keep(seq.gdn)
        self.ple = keep(seq.ple) if seq.ple is not None else None
        for j in range(g.n_qsa + 1):
            r.k_pool[j] = _p(self.k[j])
            r.v_pool[j] = _p(self.v[j])
        for j in range(g.n_qsa):
            r.idx_pooled[j] = _p(self.pooled[j])
            r.idx_tail[j] = _p(self.tail[j])
            r.idx_dead[j] = _p(self.dead[j])
            r.idx_block_pos[j] = _p(self.block_pos[j])
        r.gdn_state = _p(self.gdn)
        r.ple_hist = _p(self.ple) if self.ple is not None else None
        self.session = r


def ref_snapshot_encode(pools: RefPools, ids: np.ndarray, geom_hash: int = 0, pack_hash: int = 0) -> tuple:
    """The reference's conversation_snapshot_save + conversation_wire_encode: (payload bytes, FNV hash)."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out, n, h = C.c_void_p(), C.c_uint64(), C.c_uint64()
    err = C.create_string_buffer(512)
    rc = ref().ref_snapshot_encode(C.byref(pools.session), len(ids), _p(ids), geom_hash, pack_hash, C.byref(out),
                                   C.byref(n), C.byref(h), err, 512)
    if rc:
        raise RuntimeError(f"reference refused the snapshot ({rc}): {err.value.decode()}")
    try:
        data = (C.c_char * n.value).from_address(out.value).raw   # string_at's size is 32-bit: payloads pass 2 GiB
    finally:
        ref().ref_free(out)
    return data, h.value


def ref_decode_restore(pools: RefPools, payload: bytes) -> tuple:
    """The reference's conversation_wire_decode + conversation_snapshot_restore into `pools`: (code, message)."""
    buf = np.frombuffer(payload, dtype=np.uint8)
    err = C.create_string_buffer(512)
    rc = ref().ref_decode_restore(C.byref(pools.session), buf.ctypes.data, buf.nbytes, err, 512)
    return rc, err.value.decode()


def ref_snapshot_bytes(pools: RefPools, ids: np.ndarray) -> int:
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    n = C.c_uint64()
    err = C.create_string_buffer(512)
    rc = ref().ref_snapshot_bytes(C.byref(pools.session), len(ids), _p(ids), C.byref(n), err, 512)
    if rc:
        raise RuntimeError(err.value.decode())
    return n.value


def ref_time_wire(payload: bytes, reps: int) -> tuple:
    """The reference's conversation_wire_encode (with its streaming FNV-1a) and conversation_wire_decode of the
    image `payload` decodes to, timed `reps` times: (encode ms, decode ms) per rep."""
    buf = np.frombuffer(payload, dtype=np.uint8)
    enc = np.zeros(reps, dtype=np.float64)
    dec = np.zeros(reps, dtype=np.float64)
    err = C.create_string_buffer(512)
    rc = ref().ref_time_wire(buf.ctypes.data, buf.nbytes, reps, _p(enc), _p(dec), err, 512)
    if rc:
        raise RuntimeError(err.value.decode())
    return enc, dec


def ref_time_park_resume(src: RefPools, dst: RefPools, ids: np.ndarray, reps: int) -> tuple:
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    save = np.zeros(reps, dtype=np.float64)
    restore = np.zeros(reps, dtype=np.float64)
    err = C.create_string_buffer(512)
    rc = ref().ref_time_park_resume(C.byref(src.session), C.byref(dst.session), len(ids), _p(ids), reps, _p(save),
                                    _p(restore), err, 512)
    if rc:
        raise RuntimeError(err.value.decode())
    return save, restore
