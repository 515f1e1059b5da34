"""skv.py - Python bindings of libstrata_kv.so (the B200 KV handoff / park-resume C ABI, include/strata_kv.h).

This is the host mirror the tests and bench.py drive.  It is plumbing over the C ABI: every byte is moved by
the sm_100a kernels in csrc/skv_copy.cu.  There is no Python or CPU fallback: if the library is missing the
import of any entry point raises.

Layout of a sequence's cache in a block pool (one pool per GPU):
    slot s (block_bytes = 2 * pages_per_block * page_bytes) = [K pages 0..63][V pages 0..63] of ONE layer's
    256-token block; a page is the reference's [kv_head][page_size=4][head_dim] fp16 run
    (include/strata/kernels/qsa.hpp:178).  Layer l's logical page p of K lives at pool page
    table_l[p // 64] * 128 + p % 64 and of V at table_l[p // 64] * 128 + 64 + p % 64, which is the reference's
    QsaState::page_table format (include/strata/core/layer.hpp:220) over k_pool = pool base,
    v_pool = pool base + 64 pages.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libstrata_kv.so")

OK, EINVAL, ECUDA, ENOMEM, ETIMEOUT, EDEVICE, ERANGE = range(7)
STATUS_BAD_SRC_PAGE, STATUS_BAD_DST_PAGE, STATUS_WAIT_TIMEOUT = 0x1, 0x2, 0x4
COPY_AUTO, COPY_TMA, COPY_VEC = 0, 1, 2
PARK_DIRECT, PARK_STAGED = 1, 2
MAX_SEGMENTS = 64
NOALLOC_MAX_SEGMENTS = 512

PAGE_CELLS = 4
BLOCK_TOKENS = 256


class SkvError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"strata_kv error {code}: {message}")
        self.code = code


class Segment(C.Structure):
    _fields_ = [("src", C.c_void_p), ("dst", C.c_void_p), ("src_pages", C.c_void_p), ("dst_pages", C.c_void_p),
                ("bytes", C.c_uint64), ("page_bytes", C.c_uint32), ("reserved", C.c_uint32),
                ("src_page_limit", C.c_int64), ("dst_page_limit", C.c_int64)]


class SchedRun(C.Structure):
    """skv_sched_run: one transfer of a many-to-many hand-off batch (skv_schedule_phases)."""
    _fields_ = [("phase", C.c_int32), ("src", C.c_int32), ("lo", C.c_uint64), ("hi", C.c_uint64),
                ("wait", C.c_int32), ("signal_dst", C.c_int32), ("signal_idx", C.c_int32), ("reserved", C.c_int32)]


_lib = None

_SIGNATURES = {
    "skv_last_error": ([], C.c_char_p),
    "skv_version": ([], C.c_int),
    "skv_pool_create": ([C.c_int, C.c_int64, C.c_uint64, C.POINTER(C.c_void_p)], C.c_int),
    "skv_pool_wrap": ([C.c_int, C.c_void_p, C.c_int64, C.c_uint64, C.POINTER(C.c_void_p)], C.c_int),
    "skv_pool_destroy": ([C.c_void_p], C.c_int),
    "skv_pool_base": ([C.c_void_p], C.c_void_p),
    "skv_pool_block_bytes": ([C.c_void_p], C.c_uint64),
    "skv_pool_blocks": ([C.c_void_p], C.c_int64),
    "skv_pool_device": ([C.c_void_p], C.c_int),
    "skv_alloc_blocks": ([C.c_void_p, C.c_int64, C.c_void_p], C.c_int),
    "skv_free_blocks": ([C.c_void_p, C.c_void_p, C.c_int64], C.c_int),
    "skv_pool_free_count": ([C.c_void_p], C.c_int64),
    "skv_pool_scramble": ([C.c_void_p, C.c_uint64], C.c_int),
    "skv_expand_block_table": ([C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_void_p], C.c_int),
    "skv_copy": ([C.c_void_p, C.c_int, C.c_int, C.c_void_p], C.c_int),
    "skv_copy_noalloc": ([C.c_void_p, C.c_int, C.c_void_p, C.c_void_p], C.c_int),
    "skv_copy_gated": ([C.c_void_p, C.c_int, C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p, C.c_uint64, C.c_void_p],
                       C.c_int),
    "skv_copy_chained": ([C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p], C.c_int),
    "skv_set_copy_tuning": ([C.c_int, C.c_uint32, C.c_int, C.c_int], C.c_int),
    "skv_get_copy_tuning": ([C.POINTER(C.c_int), C.POINTER(C.c_uint32), C.POINTER(C.c_int), C.POINTER(C.c_int)], C.c_int),
    "skv_query_status": ([C.c_int, C.c_void_p, C.POINTER(C.c_uint32)], C.c_int),
    "skv_clear_status": ([C.c_int, C.c_void_p], C.c_int),
    "skv_device_initialized": ([C.c_int], C.c_int),
    "skv_host_alloc": ([C.c_uint64, C.POINTER(C.c_void_p)], C.c_int),
    "skv_host_free": ([C.c_void_p], C.c_int),
    "skv_host_register": ([C.c_void_p, C.c_uint64], C.c_int),
    "skv_host_unregister": ([C.c_void_p], C.c_int),
    "skv_park": ([C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_uint64, C.c_void_p], C.c_int),
    "skv_resume": ([C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_uint64, C.c_void_p], C.c_int),
    "skv_enable_peer": ([C.c_int, C.c_int], C.c_int),
    "skv_ipc_export": ([C.c_void_p, C.c_void_p], C.c_int),
    "skv_ipc_import": ([C.c_int, C.c_void_p, C.POINTER(C.c_void_p)], C.c_int),
    "skv_ipc_close": ([C.c_void_p], C.c_int),
    "skv_signal": ([C.c_void_p, C.c_uint64, C.c_void_p], C.c_int),
    "skv_wait_flag": ([C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p], C.c_int),
    "skv_schedule_phases": ([C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.POINTER(C.c_uint64),
                             C.POINTER(C.c_int)], C.c_int),
    "skv_slice_segments": ([C.c_void_p, C.c_int, C.c_uint64, C.c_uint64, C.c_void_p, C.c_int, C.POINTER(C.c_int)],
                           C.c_int),
}


def exported_names() -> list:
    return sorted(_SIGNATURES)


def lib() -> C.CDLL:
    """The loaded C ABI.  Raises (never falls back) when the CUDA library was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python strata-concurrent_b200/build.py` "
                               "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc:
        raise SkvError(rc, lib().skv_last_error().decode())


def _ptr(x) -> int | None:
    """A raw address from an int, a torch tensor, a numpy array or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x)}")


def _stream(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


# ------------------------------------------------------------------------------------------------ segments

def segment(src, dst, nbytes: int, *, src_pages=None, dst_pages=None, page_bytes: int = 0,
            src_page_limit: int = 0, dst_page_limit: int = 0) -> Segment:
    return Segment(_ptr(src), _ptr(dst), _ptr(src_pages), _ptr(dst_pages), int(nbytes), int(page_bytes), 0,
                   int(src_page_limit), int(dst_page_limit))


def _segment_unit(seg: Segment) -> int:
    """The granule a segment is cut on: a whole page when either side is paged, else 16 bytes."""
    unit = seg.page_bytes if (seg.src_pages or seg.dst_pages) else 16
    if unit <= 0 or seg.bytes % unit:
        raise ValueError("a segment splits on whole pages (paged) or 16-byte units (contiguous)")
    return unit


def slice_segment(seg: Segment, start: int, end: int) -> Segment:
    """Bytes [start, end) of one segment as a segment of its own; both ends must lie on the segment's granule
    (a whole page when a side is paged, 16 bytes otherwise)."""
    unit = _segment_unit(seg)
    if start % unit or end % unit or not 0 <= start < end <= seg.bytes:
        raise ValueError(f"slice [{start}, {end}) of a {seg.bytes}-byte segment is not on {unit}-byte granules")
    first_page = start // unit if (seg.src_pages or seg.dst_pages) else 0
    return Segment(
        seg.src if seg.src_pages else (seg.src or 0) + start,
        seg.dst if seg.dst_pages else (seg.dst or 0) + start,
        seg.src_pages + 4 * first_page if seg.src_pages else None,
        seg.dst_pages + 4 * first_page if seg.dst_pages else None,
        end - start, seg.page_bytes, 0, seg.src_page_limit, seg.dst_page_limit)


def split_segment(seg: Segment, max_bytes: int) -> list:
    """Cut one segment into pieces of at most `max_bytes` (whole pages for a paged side, 16-byte multiples for a
    contiguous one), in order: the pieces move exactly the bytes of the whole.  Used to pipeline a long copy
    chunk by chunk (a relay or a chained fan-out signals each piece as it lands)."""
    unit = _segment_unit(seg)
    per = max(1, max_bytes // unit) * unit
    return [slice_segment(seg, at, min(at + per, seg.bytes)) for at in range(0, seg.bytes, per)]


def slice_segments(segs: list, start: int, end: int) -> list:
    """Bytes [start, end) of a list of segments taken as one stream, in order.  A cut that falls inside a segment
    is rounded down to that segment's granule, so adjacent slices [a, b) and [b, c) always tile the stream
    exactly."""
    out, at = [], 0
    for seg in segs:
        lo, hi = max(start, at), min(end, at + seg.bytes)
        if lo < hi:
            unit = _segment_unit(seg)
            a = (lo - at) // unit * unit
            b = seg.bytes if hi == at + seg.bytes else (hi - at) // unit * unit
            if a < b:
                out.append(slice_segment(seg, a, b))
        at += seg.bytes
    return out


def copy(segs: list, engine: int = COPY_AUTO, stream=None) -> None:
    """ONE kernel launch moving every segment (gather, scatter, pool->pool, state rows, P2P, host)."""
    for i in range(0, max(len(segs), 1), MAX_SEGMENTS):
        chunk = segs[i:i + MAX_SEGMENTS]
        arr = (Segment * len(chunk))(*chunk)
        check(lib().skv_copy(arr, len(chunk), engine, _stream(stream)))


def copy_chained(segs: list, wait_flags=None, signal_flags=None, value: int = 1, timeout_ns: int = 0,
                 stream=None) -> None:
    """One TMA launch moving `segs` as a pipeline of chunks (segment c = chunk c): chunk c waits for
    wait_flags[c] >= value and, once landed, stores value to signal_flags[c] (flag arrays of 8-byte words)."""
    arr = (Segment * len(segs))(*segs)
    check(lib().skv_copy_chained(arr, len(segs), _ptr(wait_flags), _ptr(signal_flags), int(value), int(timeout_ns),
                                 _stream(stream)))


def copy_gated(segs: list, wait_flag=None, wait_value: int = 0, done_flag=None, done_value: int = 0,
               timeout_ns: int = 0, stream=None) -> None:
    """ONE TMA launch moving `segs` that first waits for *wait_flag >= wait_value and, once everything landed,
    releases done_value into *done_flag (either flag may be None)."""
    arr = (Segment * len(segs))(*segs)
    check(lib().skv_copy_gated(arr, len(segs), _ptr(wait_flag), int(wait_value), int(timeout_ns), _ptr(done_flag),
                               int(done_value), _stream(stream)))


def set_copy_tuning(tma_stages: int, tma_tile_bytes: int, tma_ctas_per_sm: int, vec_ctas_per_sm: int) -> None:
    check(lib().skv_set_copy_tuning(tma_stages, tma_tile_bytes, tma_ctas_per_sm, vec_ctas_per_sm))


def get_copy_tuning() -> tuple:
    a, b, c, d = C.c_int(), C.c_uint32(), C.c_int(), C.c_int()
    check(lib().skv_get_copy_tuning(C.byref(a), C.byref(b), C.byref(c), C.byref(d)))
    return a.value, b.value, c.value, d.value


def query_status(device: int, stream=None) -> int:
    out = C.c_uint32()
    check(lib().skv_query_status(device, _stream(stream), C.byref(out)))
    return out.value


def clear_status(device: int, stream=None) -> None:
    check(lib().skv_clear_status(device, _stream(stream)))


def park(segs: list, mode: int, staging=None, staging_bytes: int = 0, stream=None) -> None:
    arr = (Segment * len(segs))(*segs)
    check(lib().skv_park(arr, len(segs), mode, _ptr(staging), staging_bytes, _stream(stream)))


def resume(segs: list, mode: int, staging=None, staging_bytes: int = 0, stream=None) -> None:
    arr = (Segment * len(segs))(*segs)
    check(lib().skv_resume(arr, len(segs), mode, _ptr(staging), staging_bytes, _stream(stream)))


class SharedHostBuffer:
    """Pinned, device-mapped memory shared by the processes of one node: an anonymous shared-memory file (memfd)
    that the creator sizes and every user maps and registers with CUDA (skv_host_register).  `handle()` gives what
    another process needs to map the same pages: (pid, fd)."""

    def __init__(self, nbytes: int, handle: tuple | None = None):
        import mmap
        import os
        if handle is None:
            self.fd = os.memfd_create("skv-shared-host", 0)
            os.ftruncate(self.fd, nbytes)
        else:
            pid, fd = handle
            self.fd = os.open(f"/proc/{pid}/fd/{fd}", os.O_RDWR)
        self.nbytes = nbytes
        self.map = mmap.mmap(self.fd, nbytes, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
        self.ptr = C.addressof(C.c_char.from_buffer(self.map))
        check(lib().skv_host_register(self.ptr, nbytes))

    def handle(self) -> tuple:
        import os
        return (os.getpid(), self.fd)

    def close(self) -> None:
        import os
        if self.map is not None:
            check(lib().skv_host_unregister(self.ptr))
            self.ptr = 0
            self.map.close()
            os.close(self.fd)
            self.map = None


def ipc_export(dev_ptr: int) -> bytes:
    """The 64-byte CUDA IPC handle of a cudaMalloc'd allocation (its base address)."""
    h = (C.c_uint8 * 64)()
    check(lib().skv_ipc_export(dev_ptr, C.cast(h, C.c_void_p)))
    return bytes(h)


def ipc_import(device: int, handle: bytes) -> int:
    """Open a peer process's allocation on `device`; returns the mapped base address."""
    h = (C.c_uint8 * 64).from_buffer_copy(handle)
    out = C.c_void_p()
    check(lib().skv_ipc_import(device, C.cast(h, C.c_void_p), C.byref(out)))
    return out.value


def ipc_close(ptr: int) -> None:
    check(lib().skv_ipc_close(ptr))


def signal(flag: int, value: int, stream=None) -> None:
    check(lib().skv_signal(flag, value, _stream(stream)))


def wait_flag(flag: int, value: int, timeout_ns: int, stream=None) -> None:
    check(lib().skv_wait_flag(flag, value, timeout_ns, _stream(stream)))


class HostBuffer:
    """Pinned, device-mapped host memory (skv_host_alloc) with a numpy view."""

    def __init__(self, nbytes: int):
        p = C.c_void_p()
        check(lib().skv_host_alloc(nbytes, C.byref(p)))
        self.ptr = p.value or 0
        self.nbytes = nbytes
        self.array = (np.ctypeslib.as_array((C.c_uint8 * nbytes).from_address(self.ptr)) if nbytes
                      else np.zeros(0, dtype=np.uint8))

    def close(self) -> None:
        if self.ptr:
            check(lib().skv_host_free(self.ptr))
            self.ptr = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------------------------------------ the block pool

class Pool:
    """A KV block pool (skv_pool_*).  `memory` may be a caller-owned device tensor (wrapped, not freed here)."""

    def __init__(self, device: int, n_blocks: int, block_bytes: int, memory=None):
        h = C.c_void_p()
        if memory is None:
            check(lib().skv_pool_create(device, n_blocks, block_bytes, C.byref(h)))
        else:
            check(lib().skv_pool_wrap(device, _ptr(memory), n_blocks, block_bytes, C.byref(h)))
        self.handle = h.value
        self.memory = memory
        self.device = device
        self.n_blocks = n_blocks
        self.block_bytes = block_bytes

    @property
    def base(self) -> int:
        return lib().skv_pool_base(self.handle)

    def alloc(self, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.int32)
        check(lib().skv_alloc_blocks(self.handle, n, out.ctypes.data))
        return out

    def free(self, ids) -> None:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        check(lib().skv_free_blocks(self.handle, ids.ctypes.data, len(ids)))

    def free_count(self) -> int:
        return int(lib().skv_pool_free_count(self.handle))

    def scramble(self, seed: int) -> None:
        check(lib().skv_pool_scramble(self.handle, seed))

    def close(self) -> None:
        if self.handle:
            check(lib().skv_pool_destroy(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def expand_block_table(blocks, pages_per_block: int, slot_pages: int, page_offset: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.int32)
    out = np.empty(len(blocks) * pages_per_block, dtype=np.int32)
    check(lib().skv_expand_block_table(blocks.ctypes.data, len(blocks), pages_per_block, slot_pages, page_offset,
                                       out.ctypes.data))
    return out


# ------------------------------------------------------------------------------------------------ handoff plans

@dataclass
class KvGeometry:
    """The shape facts of the moved cache (include/strata/core/layout.hpp:27-60 at the configs' values)."""
    n_layers: int = 48
    qsa_interval: int = 4
    n_head_kv: int = 2
    head_dim: int = 256
    ssm_state_size: int = 128
    ssm_v_heads: int = 32
    ssm_d_conv: int = 4
    ssm_conv_channels: int = 8192

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
    def pages_per_block(self) -> int:
        return BLOCK_TOKENS // PAGE_CELLS

    @property
    def slot_pages(self) -> int:
        return 2 * self.pages_per_block

    @property
    def block_bytes(self) -> int:
        return self.slot_pages * self.page_bytes

    @property
    def gdn_bytes(self) -> int:
        s = self.ssm_state_size
        return self.n_gdn * (s * self.ssm_v_heads * s + self.ssm_conv_channels * (self.ssm_d_conv - 1)) * 4

    def pages(self, tokens: int) -> int:
        return (tokens + PAGE_CELLS - 1) // PAGE_CELLS

    def blocks(self, tokens: int) -> int:
        return (tokens + BLOCK_TOKENS - 1) // BLOCK_TOKENS

    def metric_bytes(self, tokens: int) -> int:
        return 2 * self.n_qsa * self.pages(tokens) * self.page_bytes + self.gdn_bytes + 4 * tokens


def layer_page_tables(g: KvGeometry, blocks) -> tuple:
    """(K table, V table) in pool pages for one layer's block list."""
    k = expand_block_table(blocks, g.pages_per_block, g.slot_pages, 0)
    v = expand_block_table(blocks, g.pages_per_block, g.slot_pages, g.pages_per_block)
    return k, v


class PooledSequence:
    """One sequence resident on a GPU: per-layer block tables into `pool` (device page tables in `tables`,
    an int32 device tensor [n_layers_moved, 2, pages_per_seq]), plus its GDN state rows and its token ids.
    `tables`, `gdn` and `ids` are caller-owned device buffers (any object with data_ptr(), or ints)."""

    def __init__(self, g: KvGeometry, pool: Pool, tokens: int, layers: int, blocks: np.ndarray, tables, gdn, ids):
        self.g, self.pool, self.tokens, self.layers = g, pool, tokens, layers
        self.blocks = blocks            # host copy of the block table, (layers, n_blocks) int32
        self.tables = tables
        self.gdn, self.ids = gdn, ids

    @staticmethod
    def host_tables(g: KvGeometry, blocks: np.ndarray) -> np.ndarray:
        layers, nb = blocks.shape
        out = np.empty((layers, 2, nb * g.pages_per_block), dtype=np.int32)
        for layer in range(layers):
            out[layer, 0], out[layer, 1] = layer_page_tables(g, blocks[layer])
        return out

    def table_ptr(self, layer: int, kv: int) -> int:
        per = self.g.blocks(self.tokens) * self.g.pages_per_block
        return _ptr(self.tables) + ((layer * 2 + kv) * per) * 4

    @property
    def pool_pages(self) -> int:
        return self.pool.n_blocks * self.g.slot_pages


def kv_segments_pool_to_pool(src: PooledSequence, dst: PooledSequence, dst_base=None) -> list:
    """K and V of every moved layer, source pool pages -> destination pool pages (one segment each).
    `dst_base` overrides the destination pool address (a peer mapping of the decode GPU's pool)."""
    g = src.g
    n = g.pages(src.tokens) * g.page_bytes
    base = dst.pool.base if dst_base is None else dst_base
    segs = []
    for layer in range(src.layers):
        for kv in (0, 1):
            segs.append(segment(src.pool.base, base, n, src_pages=src.table_ptr(layer, kv),
                                dst_pages=dst.table_ptr(layer, kv), page_bytes=g.page_bytes,
                                src_page_limit=src.pool_pages, dst_page_limit=dst.pool_pages))
    return segs


def state_segments(src: PooledSequence, dst_gdn, dst_ids) -> list:
    """The running state that travels with the cache: the GDN recurrent + conv rows and the token ids."""
    return [segment(src.gdn, dst_gdn, src.g.gdn_bytes), segment(src.ids, dst_ids, 16 * ((4 * src.tokens + 15) // 16))]


def image_offsets(g: KvGeometry, tokens: int, layers: int) -> dict:
    """The contiguous packed image (what a park writes): per layer K then V, then the GDN rows, then the ids,
    each 256-byte aligned."""
    n = g.pages(tokens) * g.page_bytes
    off, at = {}, 0
    for layer in range(layers):
        for kv in (0, 1):
            off[(layer, kv)] = at
            at += (n + 255) & ~255
    off["gdn"] = at
    at += (g.gdn_bytes + 255) & ~255
    off["ids"] = at
    at += (4 * tokens + 255) & ~255
    off["total"] = at
    return off


def pack_segments(src: PooledSequence, image) -> list:
    """Pool -> contiguous image (gather / pack, the B200 conversation_kv_save)."""
    g, t = src.g, src.tokens
    off = image_offsets(g, t, src.layers)
    base = _ptr(image)
    n = g.pages(t) * g.page_bytes
    segs = [segment(src.pool.base, base + off[(layer, kv)], n, src_pages=src.table_ptr(layer, kv),
                    page_bytes=g.page_bytes, src_page_limit=src.pool_pages)
            for layer in range(src.layers) for kv in (0, 1)]
    segs.append(segment(src.gdn, base + off["gdn"], g.gdn_bytes))
    segs.append(segment(src.ids, base + off["ids"], 16 * ((4 * t + 15) // 16)))
    return segs


def unpack_segments(image, dst: PooledSequence) -> list:
    """Contiguous image -> pool (scatter / unpack, the B200 conversation_kv_restore)."""
    g, t = dst.g, dst.tokens
    off = image_offsets(g, t, dst.layers)
    base = _ptr(image)
    n = g.pages(t) * g.page_bytes
    segs = [segment(base + off[(layer, kv)], dst.pool.base, n, dst_pages=dst.table_ptr(layer, kv),
                    page_bytes=g.page_bytes, dst_page_limit=dst.pool_pages)
            for layer in range(dst.layers) for kv in (0, 1)]
    segs.append(segment(base + off["gdn"], dst.gdn, g.gdn_bytes))
    segs.append(segment(base + off["ids"], dst.ids, 16 * ((4 * t + 15) // 16)))
    return segs
