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
