"""skv_copy_noalloc, the entry point for callers that cannot allocate device memory.

An engine that must not allocate on its token path (the reference's session forbids token-path
allocations, and parks and mounts happen between tokens of a running server), or that has handed all of HBM
to its block pool, calls skv_copy_noalloc instead of skv_copy.  This checks, through the C ABI, that it moves
exactly what skv_copy moves, on two calls in a row with different inputs, that its status word starts from
zero on every call, and that a plan larger than its fixed maximum is refused before anything runs.  One case is
compared with the oracle's scatter directly, and a fresh process shows that, after its warm-up call, it leaves the
device's free memory unchanged and never creates the per-device state that skv_copy allocates.

Kept in a file of its own that pytest collects last, so a stop-at-first-failure run has already run every
other test when this one runs; it builds all of its inputs itself, so it also passes alone in a fresh process.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
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


def test_noalloc_scatter_matches_the_oracle(torch_cuda):
    """A contiguous image scattered into a pool through a seed-random table: the whole pool equals the oracle's
    scatter, so pages outside the table keep their canary."""
    torch = torch_cuda
    torch.cuda.set_device(0)
    pages, pool_pages = 300, 1024
    image = np.random.default_rng(11).integers(0, 256, pages * PAGE, dtype=np.uint8)
    table = O.permutation(pool_pages, seed=12)[:pages].copy()
    expect = np.full(pool_pages * PAGE, 0x5A, dtype=np.uint8)
    O.scatter_pages(image, table, pages, PAGE, expect)
    src = torch.from_numpy(image).cuda()
    pool = torch.full((pool_pages * PAGE,), 0x5A, dtype=torch.uint8, device="cuda")
    dt = torch.from_numpy(table).cuda()
    status = torch.full((1,), 0xFF, dtype=torch.int32, device="cuda")
    seg = skv.segment(src, pool, pages * PAGE, dst_pages=dt, page_bytes=PAGE, dst_page_limit=pool_pages)
    skv.check(call_noalloc([seg], status))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert (pool.cpu().numpy() == expect).all()


FRESH_PROCESS = r"""
import sys
sys.path.insert(0, sys.argv[1])
import numpy as np
import torch
import skv
torch.cuda.set_device(0)
pages, pool_pages, page = 64, 256, 4096
src = torch.randint(0, 256, (pages * page,), dtype=torch.uint8, device="cuda")
table = torch.from_numpy(np.random.default_rng(3).permutation(pool_pages)[:pages].astype(np.int32)).cuda()
pool = torch.zeros(pool_pages * page, dtype=torch.uint8, device="cuda")
status = torch.full((1,), 7, dtype=torch.int32, device="cuda")
torch.cuda.synchronize()
L = skv.lib()
seg = (skv.Segment * 1)(skv.segment(src, pool, pages * page, dst_pages=table, page_bytes=page,
                                     dst_page_limit=pool_pages))
before = L.skv_device_initialized(0)
skv.check(L.skv_copy_noalloc(seg, 1, status.data_ptr(), None))   # the warm-up call: the one-time set-up
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info(0)[0]
for _ in range(20):
    skv.check(L.skv_copy_noalloc(seg, 1, status.data_ptr(), None))
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info(0)[0]
after = L.skv_device_initialized(0)
landed = bool(torch.equal(pool.view(pool_pages, page)[table.long()].reshape(-1), src))
print("RESULT", before, after, free0, free1, int(status.item()), int(landed))
"""


def test_noalloc_allocates_nothing_in_a_fresh_process(torch_cuda):
    """Called first in a fresh process (before any other entry point of the library): after one warm-up call, 20
    more calls leave the device's free memory exactly as it was, and the per-device state that skv_copy creates on
    first use (its status word allocation) is never created."""
    pkg = os.path.dirname(skv.__file__)
    r = subprocess.run([sys.executable, "-c", FRESH_PROCESS, pkg], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    line = next(ln for ln in r.stdout.splitlines() if ln.startswith("RESULT"))
    before, after, free0, free1, status, landed = (int(x) for x in line.split()[1:])
    assert before == 0 and after == 0, "skv_copy_noalloc created the library's per-device state"
    assert free0 == free1, f"device free memory moved by {free0 - free1} bytes across 20 calls"
    assert status == 0 and landed == 1
