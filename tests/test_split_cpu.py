"""split_segment (host logic of the pipelined relays): pieces cover exactly the whole, in order."""
import pytest

import skv


def test_paged_segment_splits_on_whole_pages():
    s = skv.segment(0x1000, 0x2000, 4096 * 10, src_pages=0x40, dst_pages=0x80, page_bytes=4096,
                    src_page_limit=99, dst_page_limit=77)
    parts = skv.split_segment(s, 3 * 4096 + 5)
    assert [p.bytes for p in parts] == [12288, 12288, 12288, 4096]
    assert [p.src_pages for p in parts] == [0x40, 0x40 + 12, 0x40 + 24, 0x40 + 36]
    assert [p.dst_pages for p in parts] == [0x80, 0x80 + 12, 0x80 + 24, 0x80 + 36]
    assert all(p.src == 0x1000 and p.dst == 0x2000 and p.page_bytes == 4096 for p in parts)
    assert all(p.src_page_limit == 99 and p.dst_page_limit == 77 for p in parts)


def test_one_paged_side_advances_the_contiguous_side():
    s = skv.segment(0x1000, 0x8000, 4096 * 4, src_pages=0x40, page_bytes=4096, src_page_limit=9)
    parts = skv.split_segment(s, 8192)
    assert [(p.src, p.dst, p.src_pages, p.dst_pages) for p in parts] == [(0x1000, 0x8000, 0x40, None),
                                                                        (0x1000, 0xA000, 0x48, None)]


def test_contiguous_segment_splits_on_16_bytes():
    parts = skv.split_segment(skv.segment(1024, 2048, 160), 50)
    assert [(p.src, p.dst, p.bytes) for p in parts] == [(1024, 2048, 48), (1072, 2096, 48), (1120, 2144, 48),
                                                        (1168, 2192, 16)]


def test_a_ragged_segment_is_refused():
    with pytest.raises(ValueError):
        skv.split_segment(skv.segment(0, 0, 4096 + 16, src_pages=8, page_bytes=4096, src_page_limit=4), 4096)


def _granules(seg):
    """Each granule a segment moves, named by where it comes from and where it goes (table entry or address)."""
    unit = seg.page_bytes if (seg.src_pages or seg.dst_pages) else 16
    out = []
    for g in range(seg.bytes // unit):
        src = ("page", seg.src, (seg.src_pages or 0) + 4 * g) if seg.src_pages else ("addr", (seg.src or 0) + g * unit)
        dst = ("page", seg.dst, (seg.dst_pages or 0) + 4 * g) if seg.dst_pages else ("addr", (seg.dst or 0) + g * unit)
        out.append((src, dst, unit))
    return out


def test_slices_of_a_segment_stream_tile_it_exactly():
    """Cut points anywhere (mid-page, mid-segment, on boundaries, repeated): the slices move every granule of the
    stream exactly once, in order, whatever the rounding inside a segment."""
    import numpy as np
    segs = [skv.segment(0x10000, 0x20000, 4096 * 7, src_pages=0x100, dst_pages=0x200, page_bytes=4096,
                        src_page_limit=50, dst_page_limit=60),
            skv.segment(0x30000, 0x40000, 160),
            skv.segment(0x50000, 0x60000, 4096 * 3, src_pages=0x300, page_bytes=4096, src_page_limit=9),
            skv.segment(0x70000, 0x80000, 16)]
    whole = [g for s in segs for g in _granules(s)]
    total = sum(s.bytes for s in segs)
    rng = np.random.default_rng(5)
    for trial in range(200):
        cuts = sorted(set([0, total] + [int(x) for x in rng.integers(0, total + 1, rng.integers(0, 8))]))
        got = []
        for a, b in zip(cuts, cuts[1:]):
            for s in skv.slice_segments(segs, a, b):
                got += _granules(s)
        assert got == whole, cuts


def test_slice_segment_refuses_cuts_off_the_granule():
    s = skv.segment(0, 0, 4096 * 4, src_pages=8, page_bytes=4096, src_page_limit=4)
    assert skv.slice_segment(s, 4096, 8192).bytes == 4096
    for a, b in ((1, 4096), (0, 4095), (4096, 4096), (0, 4096 * 5)):
        with pytest.raises(ValueError):
            skv.slice_segment(s, a, b)


def test_native_slicing_equals_slice_segments():
    """skv_slice_segments (the C ABI a C++ engine uses to cut a run's share of its flow) against slice_segments."""
    import ctypes as C
    import numpy as np
    segs = [skv.segment(0x10000, 0x20000, 4096 * 7, src_pages=0x100, dst_pages=0x200, page_bytes=4096,
                        src_page_limit=50, dst_page_limit=60),
            skv.segment(0x30000, 0x40000, 160),
            skv.segment(0x50000, 0x60000, 4096 * 3, src_pages=0x300, page_bytes=4096, src_page_limit=9),
            skv.segment(0x70000, 0x80000, 16, ),
            skv.segment(0x90000, 0xA0000, 2048 * 5, dst_pages=0x400, page_bytes=2048, dst_page_limit=8)]
    arr = (skv.Segment * len(segs))(*segs)
    total = sum(s.bytes for s in segs)
    key = lambda g: (g.src, g.dst, g.src_pages, g.dst_pages, g.bytes, g.page_bytes, g.src_page_limit,  # noqa: E731
                     g.dst_page_limit)
    rng = np.random.default_rng(9)
    out = (skv.Segment * 16)()
    n = C.c_int()
    for _ in range(300):
        lo, hi = sorted(int(x) for x in rng.integers(0, total + 1, 2))
        skv.check(skv.lib().skv_slice_segments(arr, len(segs), lo, hi, out, 16, C.byref(n)))
        assert [key(out[i]) for i in range(n.value)] == [key(g) for g in skv.slice_segments(segs, lo, hi)]
    assert skv.lib().skv_slice_segments(arr, len(segs), 0, total, out, 2, C.byref(n)) == skv.ERANGE
    assert skv.lib().skv_slice_segments(arr, len(segs), 5, 4, out, 16, C.byref(n)) == skv.EINVAL
