"""skv_copy_chained on one device: the pipelined copy of a one-to-many handoff, checked against the oracle.

A pool of seed-random pages is copied chunk by chunk (segment c = chunk c) through independent random page
tables; the oracle's gather/scatter gives the expected destination pool.  On one GPU a chained copy only ever
waits on flags that are already set when it starts (set by an earlier launch on the SAME stream, or from the
host): two launches that wait on each other never run side by side on one device.  The timeout case waits on
a flag nothing sets, with a 1 ms limit, and checks the status word and what was (not) written.
"""
import numpy as np
import pytest

import oracle as O
import skv

pytestmark = pytest.mark.gpu

PAGE = 4096


class Chunks:
    """`n_chunks` chunks of `pages` pages each: src pool pages -> dst pool pages through random tables."""

    def __init__(self, torch, n_chunks: int, pages: int, seed: int):
        self.torch = torch
        self.n, self.pages = n_chunks, pages
        total = n_chunks * pages
        self.pool_pages = total + 37                         # spare pages the tables never name
        self.src_host = O.f16_normal(self.pool_pages * PAGE // 2, seed).view(np.uint8)
        self.src_tab = O.permutation(self.pool_pages, seed + 1)[:total].copy()
        self.dst_tab = O.permutation(self.pool_pages, seed + 2)[:total].copy()
        self.src = torch.from_numpy(self.src_host.copy()).cuda()
        self.dst = torch.zeros(self.pool_pages * PAGE, dtype=torch.uint8, device="cuda")
        self.st = torch.from_numpy(self.src_tab).cuda()
        self.dt = torch.from_numpy(self.dst_tab).cuda()

    def segments(self) -> list:
        return [skv.segment(self.src, self.dst, self.pages * PAGE, src_pages=self.st.data_ptr() + 4 * c * self.pages,
                            dst_pages=self.dt.data_ptr() + 4 * c * self.pages, page_bytes=PAGE,
                            src_page_limit=self.pool_pages, dst_page_limit=self.pool_pages)
                for c in range(self.n)]

    def expected(self, chunks) -> np.ndarray:
        out = np.zeros(self.pool_pages * PAGE, dtype=np.uint8)
        for c in chunks:
            sl = slice(c * self.pages, (c + 1) * self.pages)
            image = O.gather_pages(self.src_host, self.src_tab[sl], self.pages, PAGE)
            O.scatter_pages(image, self.dst_tab[sl], self.pages, PAGE, out)
        return out

    def chunk_bytes(self, c: int) -> np.ndarray:
        """Chunk c as it lies in the destination pool, gathered through the destination table."""
        host = self.dst.cpu().numpy()
        sl = slice(c * self.pages, (c + 1) * self.pages)
        return O.gather_pages(host, self.dst_tab[sl], self.pages, PAGE)


def test_chained_copy_signals_every_chunk(torch_cuda):
    torch = torch_cuda
    ch = Chunks(torch, 6, 1024, seed=5)          # 1,536 tiles: several per CTA
    signal = torch.zeros(8, dtype=torch.int64, device="cuda")
    skv.clear_status(0)
    skv.copy_chained(ch.segments(), signal_flags=signal, value=7)
    torch.cuda.synchronize()
    assert skv.query_status(0) == 0
    assert np.array_equal(ch.dst.cpu().numpy(), ch.expected(range(6)))
    assert signal.cpu().tolist() == [7] * 6 + [0, 0]


def test_chained_copy_waits_on_flags_set_in_stream_order(torch_cuda):
    """Stage 2 of a chain: waits on the flags stage 1 stored (same stream), relays to its own flags."""
    torch = torch_cuda
    a = Chunks(torch, 5, 300, seed=11)
    mid = torch.zeros(8, dtype=torch.int64, device="cuda")
    out = torch.zeros(8, dtype=torch.int64, device="cuda")
    skv.clear_status(0)
    skv.copy_chained(a.segments(), signal_flags=mid, value=3)
    # second hop: the destination pool becomes the source of a copy into a third pool
    b_dst = torch.zeros_like(a.dst)
    segs = [skv.segment(a.dst, b_dst, a.pages * PAGE, src_pages=a.dt.data_ptr() + 4 * c * a.pages,
                        dst_pages=a.st.data_ptr() + 4 * c * a.pages, page_bytes=PAGE,
                        src_page_limit=a.pool_pages, dst_page_limit=a.pool_pages) for c in range(a.n)]
    skv.copy_chained(segs, wait_flags=mid, signal_flags=out, value=3, timeout_ns=1_000_000_000)
    torch.cuda.synchronize()
    assert skv.query_status(0) == 0
    # through dst table then back through the source table: the third pool equals the source pool on every
    # page the tables name
    got = b_dst.cpu().numpy()
    want = np.zeros_like(got)
    for c in range(a.n):
        sl = slice(c * a.pages, (c + 1) * a.pages)
        O.scatter_pages(O.gather_pages(a.src_host, a.src_tab[sl], a.pages, PAGE), a.src_tab[sl], a.pages, PAGE, want)
    assert np.array_equal(got, want)
    assert out.cpu().tolist()[:5] == [3] * 5 and mid.cpu().tolist()[:5] == [3] * 5


def test_chained_copy_split_segment_pipeline(torch_cuda):
    """One long segment cut into pieces with split_segment moves exactly what the whole would."""
    torch = torch_cuda
    ch = Chunks(torch, 1, 2048, seed=17)
    whole = ch.segments()[0]
    pieces = skv.split_segment(whole, 300 * PAGE + 123)
    assert len(pieces) == 7 and sum(p.bytes for p in pieces) == whole.bytes
    signal = torch.zeros(8, dtype=torch.int64, device="cuda")
    skv.clear_status(0)
    skv.copy_chained(pieces, signal_flags=signal, value=1)
    torch.cuda.synchronize()
    assert skv.query_status(0) == 0
    assert np.array_equal(ch.dst.cpu().numpy(), ch.expected([0]))
    assert signal.cpu().tolist()[:7] == [1] * 7


def test_chained_copy_wait_that_runs_out(torch_cuda):
    """Chunks 0-2 are released, chunk 3 never is: the wait ends after 1 ms with WAIT_TIMEOUT, chunks 0-2 are
    delivered and signalled, chunk 3 is neither read nor signalled, and the device keeps working."""
    torch = torch_cuda
    ch = Chunks(torch, 6, 512, seed=23)
    wait = torch.tensor([9, 9, 9, 0, 9, 9, 0, 0], dtype=torch.int64, device="cuda")
    signal = torch.zeros(8, dtype=torch.int64, device="cuda")
    skv.clear_status(0)
    skv.copy_chained(ch.segments(), wait_flags=wait, signal_flags=signal, value=9, timeout_ns=1_000_000)
    torch.cuda.synchronize()
    status = skv.query_status(0)
    assert status & skv.STATUS_WAIT_TIMEOUT
    sig = signal.cpu().tolist()
    assert sig[:3] == [9, 9, 9] and sig[3] == 0
    for c in range(3):
        sl = slice(c * ch.pages, (c + 1) * ch.pages)
        assert np.array_equal(ch.chunk_bytes(c), O.gather_pages(ch.src_host, ch.src_tab[sl], ch.pages, PAGE))
    assert not ch.chunk_bytes(3).any(), "a chunk whose flag never came was written"
    skv.clear_status(0)
    # the context is healthy: the same copy with every flag released completes
    wait.fill_(9)
    skv.copy_chained(ch.segments(), wait_flags=wait, signal_flags=signal, value=9, timeout_ns=1_000_000_000)
    torch.cuda.synchronize()
    assert skv.query_status(0) == 0
    assert np.array_equal(ch.dst.cpu().numpy(), ch.expected(range(6)))
