"""The NVLink hand-off between two GPUs of one process, through the C ABI, against the oracle.

The prefill GPU (cuda:0) holds a seeded synthetic cache at seed-random slots of its block pool; the decode GPU
(cuda:1) receives it at independent seed-random slots of its own pool, pre-filled with a canary byte.  Three ways
move it, each straight into the destination pool with no intermediate contiguous copy:

  pull       the decode GPU's TMA engine issues bulk loads of the prefill GPU's pool pages (peer memory, no
             multicast) and bulk stores into its own slots;
  push       the prefill GPU's vector engine stores 16-byte words into the decode GPU's slots;
  push-tma   the prefill GPU's TMA engine bulk-stores into the decode GPU's slots;
  pull-gated the pull as ONE launch (skv_copy_gated): the copy waits for READY and releases DONE itself.

The WHOLE destination pool is compared with the oracle's scatter of the same cache through the destination's
tables (tests/test_gpu_parity.py's placement), so a stray write into a slot the sequence does not own shows as a
changed canary.  The GDN rows and the ids arrive bit-exact.  Every hand-off runs the pair protocol with bounded
device-side waits: READY / DONE flags for the pull, ARRIVED for the pushes (skv_signal / skv_wait_flag), the two
sides enqueued on different GPUs so no two waiting launches share a GPU.

The reference has no peer-to-peer path (its multi-GPU hand-off goes through host RAM); the semantics matched here
are the pool layout and the page_table rule (src/kernels/cuda/qsa.cu:121-142, 405-423).
"""
import pytest

import oracle as O
import skv
from test_gpu_parity import G_FULL, G_SMALL, Placed

pytestmark = pytest.mark.gpu

WAIT_NS = 2_000_000_000   # every flag wait ends by itself after 2 s of device time
METHODS = [("pull", skv.COPY_TMA), ("push", skv.COPY_VEC), ("push-tma", skv.COPY_TMA), ("pull-gated", skv.COPY_TMA)]
PREFILL, DECODE = 0, 1


@pytest.fixture(scope="module")
def two_gpus(torch_cuda):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    skv.check(skv.lib().skv_enable_peer(DECODE, PREFILL))
    skv.check(skv.lib().skv_enable_peer(PREFILL, DECODE))
    return torch


def hand_off(torch, src: Placed, dst: Placed, method: str, engine: int, round_no: int) -> tuple:
    """One hand-off of src's whole sequence into dst's slots with the pair protocol; (prefill, decode) status."""
    flag_p = torch.zeros(1, dtype=torch.int64, device=f"cuda:{PREFILL}")   # DONE lands here
    flag_d = torch.zeros(1, dtype=torch.int64, device=f"cuda:{DECODE}")    # READY / ARRIVED land here
    skv.clear_status(PREFILL)
    skv.clear_status(DECODE)
    torch.cuda.synchronize(PREFILL)
    torch.cuda.synchronize(DECODE)
    segs = skv.kv_segments_pool_to_pool(src.ps, dst.ps) + skv.state_segments(src.ps, dst.dev_gdn, dst.dev_ids)
    L = skv.lib()
    if method == "pull-gated":
        with torch.cuda.device(DECODE):   # one launch: waits for READY, pulls, releases DONE on the prefill GPU
            skv.copy_gated(segs, flag_d.data_ptr(), round_no, flag_p.data_ptr(), round_no, timeout_ns=WAIT_NS)
        with torch.cuda.device(PREFILL):
            skv.check(L.skv_signal(flag_d.data_ptr(), round_no, None))                         # READY
            skv.check(L.skv_wait_flag(flag_p.data_ptr(), round_no, WAIT_NS, None))             # DONE
    elif method == "pull":
        with torch.cuda.device(DECODE):   # enqueue the waiting side first: it waits on the other GPU
            skv.check(L.skv_wait_flag(flag_d.data_ptr(), round_no, WAIT_NS, None))            # READY
            skv.copy(segs, engine)                                                             # loads over NVLink
            skv.check(L.skv_signal(flag_p.data_ptr(), round_no, None))                         # DONE
        with torch.cuda.device(PREFILL):
            skv.check(L.skv_signal(flag_d.data_ptr(), round_no, None))                         # READY
            skv.check(L.skv_wait_flag(flag_p.data_ptr(), round_no, WAIT_NS, None))             # DONE
    else:
        with torch.cuda.device(DECODE):
            skv.check(L.skv_wait_flag(flag_d.data_ptr(), round_no, WAIT_NS, None))            # ARRIVED
        with torch.cuda.device(PREFILL):
            skv.copy(segs, engine)                                                             # stores over NVLink
            skv.check(L.skv_signal(flag_d.data_ptr(), round_no, None))                         # ARRIVED
    torch.cuda.synchronize(PREFILL)
    torch.cuda.synchronize(DECODE)
    assert int(flag_d.item()) == round_no
    if method.startswith("pull"):
        assert int(flag_p.item()) == round_no
    return skv.query_status(PREFILL), skv.query_status(DECODE)


def check_landed(torch, seq: O.Sequence, dst: Placed) -> None:
    got = dst.dev_pool.cpu().numpy()
    assert (got == dst.expected_pool(seq)).all(), "destination pool differs from the oracle's scatter"
    assert (dst.dev_gdn.cpu().numpy() == seq.gdn).all()
    assert (dst.dev_ids.cpu().numpy()[:seq.tokens] == seq.ids).all()


@pytest.fixture(scope="module")
def config1_on_prefill(two_gpus):
    """Config 1's cache (4,096 tokens, 12 full-geometry layers) at seed-random slots of a 4,096-block pool on the
    prefill GPU, placed once for the module."""
    seq = O.make_sequence(G_FULL, 4096, seed=1)
    return seq, Placed(two_gpus, G_FULL, seq, 4096, seed=11, layers=G_FULL.n_qsa, device=PREFILL)


@pytest.mark.parametrize("method,engine", METHODS, ids=[m for m, _ in METHODS])
def test_config1_hand_off_between_two_gpus(two_gpus, config1_on_prefill, method, engine):
    """Config 1 handed to independent random slots of the decode GPU's 1,024-block pool."""
    torch = two_gpus
    seq, src = config1_on_prefill
    dst = Placed(torch, G_FULL, seq, 1024, seed=23, layers=G_FULL.n_qsa, canary=0xA5, upload=False, device=DECODE)
    assert hand_off(torch, src, dst, method, engine, 1) == (0, 0)
    check_landed(torch, seq, dst)


@pytest.mark.parametrize("method,engine", METHODS, ids=[m for m, _ in METHODS])
@pytest.mark.parametrize("t", [1, 257, 2048])
def test_ragged_lengths_between_two_gpus(two_gpus, method, engine, t):
    """Partial pages, a block boundary plus one token, and several whole blocks (plus the draft-like extra
    layer), each handed over three times in a row through the same flags' rising values."""
    torch = two_gpus
    layers = G_SMALL.n_qsa + 1
    seq = O.make_sequence(G_SMALL, t, seed=t)
    src = Placed(torch, G_SMALL, seq, 96, seed=t + 1, layers=layers, device=PREFILL)
    dst = Placed(torch, G_SMALL, seq, 96, seed=t + 2, layers=layers, canary=0x5A, upload=False, device=DECODE)
    for r in (1, 2, 3):
        assert hand_off(torch, src, dst, method, engine, r) == (0, 0)
    check_landed(torch, seq, dst)


def test_pull_refuses_an_out_of_pool_source_page(two_gpus):
    """A source table entry outside the prefill GPU's pool is never dereferenced over the link: the page is
    skipped, the decode GPU's status says so, and every other page still lands."""
    torch = two_gpus
    pb, pages, limit = 4096, 40, 64
    src = torch.randint(0, 256, (limit * pb,), dtype=torch.uint8, device=f"cuda:{PREFILL}")
    table = O.permutation(limit, seed=9)[:pages].copy()
    table[5] = limit + 77
    st = torch.from_numpy(table).to(f"cuda:{DECODE}")
    out = torch.zeros(pages * pb, dtype=torch.uint8, device=f"cuda:{DECODE}")
    skv.clear_status(DECODE)
    with torch.cuda.device(DECODE):
        skv.copy([skv.segment(src, out, pages * pb, src_pages=st, page_bytes=pb, src_page_limit=limit)], skv.COPY_TMA)
    torch.cuda.synchronize(DECODE)
    assert skv.query_status(DECODE) == skv.STATUS_BAD_SRC_PAGE
    s = src.view(limit, pb).cpu().numpy()
    o = out.view(pages, pb).cpu().numpy()
    for i in range(pages):
        assert (o[i] == (0 if i == 5 else s[table[i]])).all()


def test_wait_for_a_peer_that_never_signals_times_out(two_gpus):
    """The decode GPU waits for a READY the prefill GPU never raises: the wait ends after its limit with the
    timeout bit, the copy after it still runs (its source is ready), and both contexts keep working."""
    torch = two_gpus
    flag = torch.zeros(1, dtype=torch.int64, device=f"cuda:{DECODE}")
    a = torch.arange(4096, dtype=torch.int32, device=f"cuda:{PREFILL}")
    b = torch.zeros(4096, dtype=torch.int32, device=f"cuda:{DECODE}")
    skv.clear_status(DECODE)
    with torch.cuda.device(DECODE):
        skv.check(skv.lib().skv_wait_flag(flag.data_ptr(), 1, 20_000_000, None))
        skv.copy([skv.segment(a, b, a.numel() * 4)], skv.COPY_TMA)
    torch.cuda.synchronize(DECODE)
    assert skv.query_status(DECODE) == skv.STATUS_WAIT_TIMEOUT
    assert torch.equal(a.cpu(), b.cpu())
