"""skv_copy_noalloc, the entry point for callers that cannot allocate device memory.

An engine that must not allocate on its token path (the reference's session forbids token-path
allocations, and parks and mounts happen between tokens of a running server), or that has handed all of HBM
to its block pool, calls skv_copy_noalloc instead of skv_copy.  This checks, through the C ABI, that it moves
exactly what skv_copy moves, on two calls in a row with different inputs, that its status word starts from
zero on every call, and that a plan larger than its fixed maximum is refused before anything runs.

Kept in a file of its own that pytest collects last, so a stop-at-first-failure run has already run every
other test when this one runs; it builds all of its inputs itself, so it also passes alone in a fresh process.
"""
import numpy as np
import pytest

import skv

pytestmark = pytest.mark.gpu

PAGE = 4096


def seq_case(torch, seed: int, layers: int, pages: int, pool_pages: int):
    """A source pool with random bytes, per-layer random source and destination page tables, and the segment
    list that moves every layer (one segment per layer) plus one contiguous state segment."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    rng = np.random.default_rng(seed)
    src_pool = torch.randint(0, 256, (pool_pages * PAGE,), generator=gen, dtype=torch.uint8, device="cuda")
    state = torch.randint(0, 256, (1 << 20,), generator=gen, dtype=torch.uint8, device="cuda")
    src_tab = torch.from_numpy(np.stack([rng.permutation(pool_pages)[:pages] for _ in range(layers)]).astype(np.int32)).cuda()
    # destination pages are disjoint across layers, as slots handed out by one pool are
    dst_tab = torch.from_numpy(rng.permutation(pool_pages)[:layers * pages].reshape(layers, pages).astype(np.int32)).cuda()
    return src_pool, state, src_tab, dst_tab


def segments(src_pool, state, src_tab, dst_tab, dst_pool, dst_state, pool_pages):
    pages = src_tab.shape[1]
    segs = [skv.segment(src_pool, dst_pool, pages * PAGE, src_pages=src_tab[i], dst_pages=dst_tab[i], page_bytes=PAGE,
                        src_page_limit=pool_pages, dst_page_limit=pool_pages) for i in range(src_tab.shape[0])]
    segs.append(skv.segment(state, dst_state, state.numel()))
    return segs


def call_noalloc(segs, status):
    arr = (skv.Segment * len(segs))(*segs)
    return skv.lib().skv_copy_noalloc(arr, len(segs), status.data_ptr(), None)


def test_noalloc_matches_skv_copy_on_two_calls_in_a_row(torch_cuda):
    torch = torch_cuda
    torch.cuda.set_device(0)
    pool_pages = 2048
    status = torch.full((1,), 0xFFFF, dtype=torch.int32, device="cuda")

    # call 1: 24 layers, one destination table entry outside the pool (skipped and flagged by both paths)
    src_pool, state, src_tab, dst_tab = seq_case(torch, 1, layers=24, pages=40, pool_pages=pool_pages)
    dst_tab[5, 17] = pool_pages + 3
    want_pool = torch.zeros(pool_pages * PAGE, dtype=torch.uint8, device="cuda")
    want_state = torch.zeros_like(state)
    got_pool, got_state = torch.zeros_like(want_pool), torch.zeros_like(want_state)
    skv.clear_status(0)
    skv.copy(segments(src_pool, state, src_tab, dst_tab, want_pool, want_state, pool_pages), skv.COPY_VEC)
    skv.check(call_noalloc(segments(src_pool, state, src_tab, dst_tab, got_pool, got_state, pool_pages), status))
    torch.cuda.synchronize()
    assert skv.query_status(0) == skv.STATUS_BAD_DST_PAGE
    assert int(status.item()) == skv.STATUS_BAD_DST_PAGE
    assert torch.equal(got_pool, want_pool) and torch.equal(got_state, want_state)

    # call 2, right after: different inputs and 100 segments (more than skv_copy takes in one launch);
    # the status word must start from zero again
    src_pool, state, src_tab, dst_tab = seq_case(torch, 2, layers=99, pages=5, pool_pages=pool_pages)
    want_pool = torch.zeros(pool_pages * PAGE, dtype=torch.uint8, device="cuda")
    want_state = torch.zeros_like(state)
    got_pool, got_state = torch.zeros_like(want_pool), torch.zeros_like(want_state)
    segs_want = segments(src_pool, state, src_tab, dst_tab, want_pool, want_state, pool_pages)
    segs_got = segments(src_pool, state, src_tab, dst_tab, got_pool, got_state, pool_pages)
    assert len(segs_got) == 100
    skv.clear_status(0)
    skv.copy(segs_want, skv.COPY_VEC)
    skv.check(call_noalloc(segs_got, status))
    torch.cuda.synchronize()
    assert skv.query_status(0) == 0 and int(status.item()) == 0
    assert torch.equal(got_pool, want_pool) and torch.equal(got_state, want_state)
    assert int(got_pool.count_nonzero()) > 0


def test_noalloc_refuses_plans_beyond_its_maximum(torch_cuda):
    torch = torch_cuda
    a = torch.zeros(16, dtype=torch.uint8, device="cuda")
    segs = [skv.segment(a, a, 16)] * (skv.NOALLOC_MAX_SEGMENTS + 1)
    arr = (skv.Segment * len(segs))(*segs)
    rc = skv.lib().skv_copy_noalloc(arr, len(segs), None, None)
    assert rc == skv.ERANGE
    assert "maximum" in skv.lib().skv_last_error().decode()
    torch.cuda.synchronize()
