"""The streaming-residency oracle (orc_stream_resolve, the checker the GPU resolve is compared with bit for bit)
against the policy's own invariants, over long random call sequences on CPU.

After every call: the page table and the slot map agree both ways and no claim (-2) is left behind; every block the
call looked up is resident unless the call reported that it could not place every miss; a block that was already
resident keeps its slot (hits never move); every slot the call used carries the call's epoch and its reference
bit; and the counters and the return value count what happened.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O

STEP_COUNT, STEP_WIDTH, CTL_INTS = 4, 3, 16


def _resolve(state, ids, steps, n_q, cap, page_size):
    table, sb, st, rf, ctl = state
    n_blocks, n_slots = len(table), len(sb)
    mb = np.zeros(max(n_slots, 1), dtype=np.int32)
    ms = np.zeros(max(n_slots, 1), dtype=np.int32)
    p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    L = O.lib()
    L.orc_stream_resolve.restype = C.c_int64
    L.orc_stream_resolve.argtypes = [C.c_void_p] * 7 + [C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_int64,
                                                        C.c_int64, C.c_int64]
    return L.orc_stream_resolve(p(table), p(sb), p(st), p(rf), p(ctl), p(mb), p(ms), n_blocks, n_slots, p(ids), p(steps),
                                n_q, cap, page_size)


@pytest.mark.parametrize("n_blocks,n_slots,seed", [(64, 16, 1), (40, 40, 2), (200, 7, 3), (16, 1, 4)])
def test_resolve_keeps_the_policy_invariants(n_blocks, n_slots, seed):
    rng = np.random.default_rng(seed)
    page_size, cap = 4, 48
    table = np.full(n_blocks, -1, dtype=np.int32)
    sb = np.full(n_slots, -1, dtype=np.int32)
    st = np.full(n_slots, -1, dtype=np.int32)
    rf = np.zeros(n_slots, dtype=np.int32)
    ctl = np.zeros(CTL_INTS, dtype=np.int32)
    state = (table, sb, st, rf, ctl)
    for call in range(300):
        n_q = int(rng.integers(1, 4))
        ids = np.zeros((n_q, cap), dtype=np.int32)
        steps = np.zeros((n_q, STEP_COUNT), dtype=np.int32)
        looked = set()
        for q in range(n_q):
            width = int(rng.integers(0, cap + 1))
            # ascending token positions (the selection), mostly inside the table, a few outside it
            pos = np.sort(rng.choice(n_blocks * page_size + 8, size=width, replace=False)).astype(np.int32)
            ids[q, :width] = pos
            steps[q, STEP_WIDTH] = width
            looked |= {int(x) // page_size for x in pos if int(x) // page_size < n_blocks}
        before_table = table.copy()
        calls_before = int(ctl[4:10].view(np.uint64)[2])
        ctl[3] = 0
        placed = _resolve(state, ids, steps, n_q, cap, page_size)
        epoch = int(ctl[0])
        # the map agrees both ways, and no claim is left
        assert (table >= -1).all()
        for s in range(n_slots):
            if sb[s] >= 0:
                assert table[sb[s]] == s
        for b in np.nonzero(table >= 0)[0]:
            assert sb[table[b]] == b
        # hits never move; looked-up blocks are resident unless the call could not place every miss
        for b in looked:
            if before_table[b] >= 0:
                assert table[b] == before_table[b]
            if table[b] >= 0:
                assert st[table[b]] == epoch and rf[table[b]] == 1
            else:
                assert ctl[3] == 1
        # the return value is the number of new placements, and only looked-up blocks were placed
        new = {int(b) for b in np.nonzero((table >= 0) & (before_table < 0))[0]}
        assert placed == len(new) and new <= looked
        assert int(ctl[4:10].view(np.uint64)[2]) == calls_before + 1
