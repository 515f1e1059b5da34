"""Parity of the sm_100a path against the oracle, through the C ABI.

Every case places a seeded synthetic cache into a block pool at seed-random slots (the placement is done
on the host by the ORACLE's scatter and uploaded whole), runs ONE skv_copy launch, reads the result back
and compares bytes: bit-exact, no tolerance (this path is byte movement).  Config 1's blobs are also
checked against the FNV-1a hashes the reference itself produced (tests/golden/golden.json).
"""
import json
import os

import numpy as np
import pytest

import oracle as O
import skv

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.json")
ENGINES = [skv.COPY_TMA, skv.COPY_VEC]
G_FULL = O.Geometry()
G_SMALL = O.Geometry(n_layers=8, qsa_interval=4, n_head_kv=2, head_dim=256, ssm_state_size=8, ssm_v_heads=4,
                     ssm_conv_channels=64, idx_key_dim=8)


def kvg(g: O.Geometry) -> skv.KvGeometry:
    return skv.KvGeometry(n_layers=g.n_layers, qsa_interval=g.qsa_interval, n_head_kv=g.n_head_kv,
                          head_dim=g.head_dim, ssm_state_size=g.ssm_state_size, ssm_v_heads=g.ssm_v_heads,
                          ssm_d_conv=g.ssm_d_conv, ssm_conv_channels=g.ssm_conv_channels)


class Placed:
    """A Sequence placed into a pool: host mirror of the whole pool + device copy + the PooledSequence."""

    def __init__(self, torch, g: O.Geometry, seq: O.Sequence, n_blocks: int, seed: int, layers: int,
                 canary: int = 0, upload: bool = True, device: int = 0):
        self.torch = torch
        self.device = device
        where = f"cuda:{device}"
        self.kg = kg = kvg(g)
        self.host_pool = np.full(n_blocks * kg.block_bytes, canary, dtype=np.uint8)
        self.dev_pool = torch.empty(n_blocks * kg.block_bytes, dtype=torch.uint8, device=where)
        self.pool = skv.Pool(device, n_blocks, kg.block_bytes, memory=self.dev_pool)
        self.pool.scramble(seed)
        nb = kg.blocks(seq.tokens)
        self.blocks = np.stack([self.pool.alloc(nb) for _ in range(layers)]) if layers else np.zeros((0, nb), np.int32)
        tables = skv.PooledSequence.host_tables(kg, self.blocks)
        pages = kg.pages(seq.tokens)
        for layer in range(layers):
            k_table = O.expand_block_table(self.blocks[layer], kg.pages_per_block, kg.slot_pages, 0)
            v_table = O.expand_block_table(self.blocks[layer], kg.pages_per_block, kg.slot_pages, kg.pages_per_block)
            assert (tables[layer, 0] == k_table).all() and (tables[layer, 1] == v_table).all()
            if upload:
                O.scatter_pages(seq.k[layer], k_table, pages, kg.page_bytes, self.host_pool)
                O.scatter_pages(seq.v[layer], v_table, pages, kg.page_bytes, self.host_pool)
        self.dev_pool.copy_(torch.from_numpy(self.host_pool))
        self.dev_tables = torch.from_numpy(tables.reshape(-1).copy()).to(where)
        ids_pad = np.zeros(((4 * seq.tokens + 15) // 16) * 4, dtype=np.int32)
        ids_pad[:seq.tokens] = seq.ids if upload else 0
        self.dev_gdn = torch.from_numpy(seq.gdn.copy() if upload else np.zeros_like(seq.gdn)).to(where)
        self.dev_ids = torch.from_numpy(ids_pad).to(where)
        self.ps = skv.PooledSequence(kg, self.pool, seq.tokens, layers, self.blocks, self.dev_tables, self.dev_gdn,
                                     self.dev_ids)
        torch.cuda.synchronize(device)

    def expected_pool(self, seq: O.Sequence) -> np.ndarray:
        """This pool as the oracle writes it: the host mirror with every layer of `seq` scattered through THIS
        placement's block tables (slots the sequence does not own keep their canary)."""
        kg = self.kg
        expect = self.host_pool.copy()
        for j in range(len(self.blocks)):
            kt, vt = skv.layer_page_tables(kg, self.blocks[j])
            O.scatter_pages(seq.k[j], kt, kg.pages(seq.tokens), kg.page_bytes, expect)
            O.scatter_pages(seq.v[j], vt, kg.pages(seq.tokens), kg.page_bytes, expect)
        return expect


def run(torch, segs, engine):
    skv.clear_status(0)
    skv.copy(segs, engine)
    torch.cuda.synchronize()
    return skv.query_status(0)


def to_host(t):
    return t.cpu().numpy()


def image_blob(img: np.ndarray, off: dict, key, n: int) -> np.ndarray:
    return img[off[key]:off[key] + n]


@pytest.mark.parametrize("engine", ENGINES)
def test_pack_config1_matches_reference_blobs(torch_cuda, engine):
    """Config 1: 4,096 tokens at seed-random slots of a 4,096-block pool; the GPU gather equals the K/V the
    reference's conversation_kv_save wrote from its identity pool, blob by blob (FNV-1a from the golden
    fixture) and byte by byte (oracle)."""
    torch = torch_cuda
    golden = json.load(open(GOLDEN))["config1"]
    t = golden["tokens"]
    seq = O.make_sequence(G_FULL, t, seed=golden["seed"])
    src = Placed(torch, G_FULL, seq, 4096, seed=11, layers=G_FULL.n_qsa)
    kg = src.kg
    off = skv.image_offsets(kg, t, G_FULL.n_qsa)
    image = torch.zeros(off["total"], dtype=torch.uint8, device="cuda")
    assert run(torch, skv.pack_segments(src.ps, image), engine) == 0
    img = to_host(image)
    n = kg.pages(t) * kg.page_bytes
    for j in range(G_FULL.n_qsa):
        k, v = image_blob(img, off, (j, 0), n), image_blob(img, off, (j, 1), n)
        assert (k == seq.k[j]).all() and (v == seq.v[j]).all()
        assert [n, O.fnv1a64(k)] == golden["blobs"]["kv"][j]["k"]
        assert [n, O.fnv1a64(v)] == golden["blobs"]["kv"][j]["v"]
    gdn = image_blob(img, off, "gdn", kg.gdn_bytes)
    assert [kg.gdn_bytes, O.fnv1a64(gdn)] == golden["blobs"]["live"]["gdn"]
    assert O.fnv1a64(image_blob(img, off, "ids", 4 * t)) == golden["blobs"]["live"]["ids"]


@pytest.mark.parametrize("engine", ENGINES)
def test_unpack_config1_into_a_different_table(torch_cuda, engine):
    """The scatter writes exactly the oracle's pool: every placed page, and not one byte elsewhere (the
    untouched slots keep their canary)."""
    torch = torch_cuda
    t = 4096
    seq = O.make_sequence(G_FULL, t, seed=1)
    dst = Placed(torch, G_FULL, seq, 1024, seed=23, layers=G_FULL.n_qsa, canary=0xA5, upload=False)
    kg = dst.kg
    off = skv.image_offsets(kg, t, G_FULL.n_qsa)
    host_img = np.zeros(off["total"], dtype=np.uint8)
    n = kg.pages(t) * kg.page_bytes
    for j in range(G_FULL.n_qsa):
        host_img[off[(j, 0)]:off[(j, 0)] + n] = seq.k[j]
        host_img[off[(j, 1)]:off[(j, 1)] + n] = seq.v[j]
    host_img[off["gdn"]:off["gdn"] + kg.gdn_bytes] = seq.gdn.view(np.uint8)
    host_img[off["ids"]:off["ids"] + 4 * t] = seq.ids.view(np.uint8)
    image = torch.from_numpy(host_img).cuda()
    assert run(torch, skv.unpack_segments(image, dst.ps), engine) == 0
    expect = dst.host_pool.copy()
    for j in range(G_FULL.n_qsa):
        per = kg.blocks(t) * kg.pages_per_block
        kt = to_host(dst.dev_tables)[(2 * j) * per:(2 * j + 1) * per]
        vt = to_host(dst.dev_tables)[(2 * j + 1) * per:(2 * j + 2) * per]
        O.scatter_pages(seq.k[j], kt, kg.pages(t), kg.page_bytes, expect)
        O.scatter_pages(seq.v[j], vt, kg.pages(t), kg.page_bytes, expect)
    assert (to_host(dst.dev_pool) == expect).all()
    assert (to_host(dst.dev_gdn) == seq.gdn).all()
    assert (to_host(dst.dev_ids)[:t] == seq.ids).all()


@pytest.mark.parametrize("engine", ENGINES)
@pytest.mark.parametrize("t", [1, 3, 4, 5, 255, 256, 257, 1000, 2048])
def test_pool_to_pool_edge_lengths(torch_cuda, engine, t):
    """Config 2a's operation (pool -> pool with an independent random table) at ragged lengths: partial
    pages, partial blocks, block boundaries.  The whole destination pool must equal the oracle's."""
    torch = torch_cuda
    layers = G_SMALL.n_qsa + 1
    seq = O.make_sequence(G_SMALL, t, seed=t)
    src = Placed(torch, G_SMALL, seq, 96, seed=t + 1, layers=layers)
    dst = Placed(torch, G_SMALL, seq, 96, seed=t + 2, layers=layers, canary=0x5A, upload=False)
    kg = src.kg
    gdn_out = torch.zeros_like(dst.dev_gdn)
    ids_out = torch.zeros_like(dst.dev_ids)
    segs = skv.kv_segments_pool_to_pool(src.ps, dst.ps) + skv.state_segments(src.ps, gdn_out, ids_out)
    assert run(torch, segs, engine) == 0
    expect = dst.host_pool.copy()
    pages = kg.pages(t)
    for j in range(layers):
        kt, vt = skv.layer_page_tables(kg, dst.blocks[j])
        O.scatter_pages(seq.k[j], kt, pages, kg.page_bytes, expect)
        O.scatter_pages(seq.v[j], vt, pages, kg.page_bytes, expect)
    assert (to_host(dst.dev_pool) == expect).all()
    assert (to_host(gdn_out) == seq.gdn).all() and (to_host(ids_out)[:t] == seq.ids).all()


@pytest.mark.slow
@pytest.mark.parametrize("engine", ENGINES)
def test_pool_to_pool_32k_round_trip(torch_cuda, engine):
    """Config 2a at full size (32,768 tokens, 128 blocks/layer, 12 layers): size-independent properties.
    The destination read back through ITS table equals the source read through ITS table, equals the data
    that was placed; page checksums of the two agree."""
    torch = torch_cuda
    kg = skv.KvGeometry()
    t, n_blocks = 32768, 4096
    pages = kg.pages(t)
    gen = torch.Generator(device="cuda").manual_seed(5)
    src_mem = torch.zeros(n_blocks * kg.block_bytes, dtype=torch.uint8, device="cuda")
    dst_mem = torch.zeros_like(src_mem)
    src_pool = skv.Pool(0, n_blocks, kg.block_bytes, memory=src_mem)
    dst_pool = skv.Pool(0, n_blocks, kg.block_bytes, memory=dst_mem)
    src_pool.scramble(101)
    dst_pool.scramble(202)
    sb = np.stack([src_pool.alloc(kg.blocks(t)) for _ in range(kg.n_qsa)])
    db = np.stack([dst_pool.alloc(kg.blocks(t)) for _ in range(kg.n_qsa)])
    st = torch.from_numpy(skv.PooledSequence.host_tables(kg, sb).reshape(-1).copy()).cuda()
    dt = torch.from_numpy(skv.PooledSequence.host_tables(kg, db).reshape(-1).copy()).cuda()
    logical = torch.randn(kg.n_qsa, 2, pages, kg.page_bytes // 2, generator=gen, device="cuda",
                          dtype=torch.float16).view(torch.uint8)
    page_view = src_mem.view(-1, kg.page_bytes)
    tab = st.view(kg.n_qsa, 2, -1)[:, :, :pages].long()
    page_view[tab.reshape(-1)] = logical.reshape(-1, kg.page_bytes)
    gdn = torch.randn(kg.gdn_bytes // 4, generator=gen, device="cuda") * 0.02
    ids = torch.randint(0, 151936, (t,), generator=gen, device="cuda", dtype=torch.int32)
    gdn_out, ids_out = torch.zeros_like(gdn), torch.zeros_like(ids)
    src = skv.PooledSequence(kg, src_pool, t, kg.n_qsa, sb, st, gdn, ids)
    dst = skv.PooledSequence(kg, dst_pool, t, kg.n_qsa, db, dt, gdn_out, ids_out)
    segs = skv.kv_segments_pool_to_pool(src, dst) + skv.state_segments(src, gdn_out, ids_out)
    assert run(torch, segs, engine) == 0
    back = dst_mem.view(-1, kg.page_bytes)[dt.view(kg.n_qsa, 2, -1)[:, :, :pages].long().reshape(-1)]
    assert torch.equal(back, logical.reshape(-1, kg.page_bytes))
    assert torch.equal(gdn_out, gdn) and torch.equal(ids_out, ids)
    # slots the sequence does not own are untouched
    untouched = np.setdiff1d(np.arange(n_blocks), db.reshape(-1))[:64]
    assert int(dst_mem.view(n_blocks, -1)[torch.from_numpy(untouched).cuda().long()].abs().sum()) == 0
    host_a = back.cpu().numpy()
    assert O.page_checksum(host_a, kg.page_bytes) == O.page_checksum(logical.cpu().numpy(), kg.page_bytes)


@pytest.mark.slow
def test_pool_to_pool_32k_matches_the_reference_blobs(torch_cuda):
    """Config 2(a) at full size, pinned to the reference: the oracle's 32,768-token sequence (seed 2) placed at
    seed-random slots of a 4,096-block pool, handed pool -> pool into an independent random table of a second pool
    (ONE TMA-engine launch), then packed out of the DESTINATION through its table: every layer's K and V, the GDN
    rows and the ids hash (FNV-1a) to what the reference's own conversation_snapshot_save wrote for the same
    sequence (tests/golden/golden.json config2a_32k), and the destination's unowned slots keep their canary."""
    torch = torch_cuda
    golden = json.load(open(GOLDEN))["config2a_32k"]
    t = golden["tokens"]
    layers = G_FULL.n_qsa + 1   # the draft layer too, as the reference saves it
    seq = O.make_sequence(G_FULL, t, seed=golden["seed"])
    src = Placed(torch, G_FULL, seq, 4096, seed=31, layers=layers)
    dst = Placed(torch, G_FULL, seq, 4096, seed=47, layers=layers, canary=0x3C, upload=False)
    kg = src.kg
    segs = skv.kv_segments_pool_to_pool(src.ps, dst.ps) + skv.state_segments(src.ps, dst.dev_gdn, dst.dev_ids)
    assert run(torch, segs, skv.COPY_TMA) == 0
    del src
    off = skv.image_offsets(kg, t, layers)
    image = torch.zeros(off["total"], dtype=torch.uint8, device="cuda")
    assert run(torch, skv.pack_segments(dst.ps, image), skv.COPY_TMA) == 0
    img = to_host(image)
    n = kg.pages(t) * kg.page_bytes
    for j in range(layers):
        assert [n, O.fnv1a64(image_blob(img, off, (j, 0), n))] == golden["blobs"]["kv"][j]["k"]
        assert [n, O.fnv1a64(image_blob(img, off, (j, 1), n))] == golden["blobs"]["kv"][j]["v"]
    assert [kg.gdn_bytes, O.fnv1a64(image_blob(img, off, "gdn", kg.gdn_bytes))] == golden["blobs"]["live"]["gdn"]
    assert O.fnv1a64(image_blob(img, off, "ids", 4 * t)) == golden["blobs"]["live"]["ids"]
    owned = np.zeros(4096, dtype=bool)
    owned[dst.blocks.reshape(-1)] = True
    pool = to_host(dst.dev_pool).reshape(4096, -1)
    assert (pool[~owned] == 0x3C).all()


@pytest.mark.parametrize("mode", [skv.PARK_DIRECT, skv.PARK_STAGED])
def test_park_resume_pinned_host(torch_cuda, mode):
    """Config 2b: park to pinned host memory, resume into a different table; both ends bit-exact."""
    torch = torch_cuda
    t = 1000
    layers = G_SMALL.n_qsa + 1
    seq = O.make_sequence(G_SMALL, t, seed=77)
    src = Placed(torch, G_SMALL, seq, 64, seed=1, layers=layers)
    dst = Placed(torch, G_SMALL, seq, 64, seed=2, layers=layers, upload=False)
    kg = src.kg
    off = skv.image_offsets(kg, t, layers)
    host = skv.HostBuffer(off["total"])
    staging = torch.empty(off["total"] + 256 * 64, dtype=torch.uint8, device="cuda")
    skv.clear_status(0)
    skv.park(skv.pack_segments(src.ps, host.ptr), mode, staging, staging.numel())
    torch.cuda.synchronize()
    n = kg.pages(t) * kg.page_bytes
    for j in range(layers):
        assert (host.array[off[(j, 0)]:off[(j, 0)] + n] == seq.k[j]).all()
        assert (host.array[off[(j, 1)]:off[(j, 1)] + n] == seq.v[j]).all()
    assert (host.array[off["gdn"]:off["gdn"] + kg.gdn_bytes] == seq.gdn.view(np.uint8)).all()
    skv.resume(skv.unpack_segments(host.ptr, dst.ps), mode, staging, staging.numel())
    torch.cuda.synchronize()
    assert skv.query_status(0) == 0
    expect = dst.host_pool.copy()
    for j in range(layers):
        kt, vt = skv.layer_page_tables(kg, dst.blocks[j])
        O.scatter_pages(seq.k[j], kt, kg.pages(t), kg.page_bytes, expect)
        O.scatter_pages(seq.v[j], vt, kg.pages(t), kg.page_bytes, expect)
    assert (to_host(dst.dev_pool) == expect).all()
    assert (to_host(dst.dev_gdn) == seq.gdn).all()
    host.close()


@pytest.mark.parametrize("engine", ENGINES)
def test_out_of_pool_table_entry_is_refused_on_device(torch_cuda, engine):
    """A table entry outside the pool is never dereferenced: the page is skipped, the status word says so,
    and every other page still arrives."""
    torch = torch_cuda
    pb, pages, limit = 4096, 40, 64
    src = torch.randint(0, 256, (pages * pb,), dtype=torch.uint8, device="cuda")
    pool = torch.zeros(limit * pb, dtype=torch.uint8, device="cuda")
    table = O.permutation(limit, seed=4)[:pages].copy()
    table[17] = limit + 1000
    dt = torch.from_numpy(table).cuda()
    seg = skv.segment(src, pool, pages * pb, dst_pages=dt, page_bytes=pb, dst_page_limit=limit)
    assert run(torch, [seg], engine) == skv.STATUS_BAD_DST_PAGE
    p = pool.view(limit, pb).cpu().numpy()
    s = src.view(pages, pb).cpu().numpy()
    for i in range(pages):
        if i != 17:
            assert (p[table[i]] == s[i]).all()


def test_small_page_granule_vector_engine(torch_cuda):
    """int8 scale pages are 64 bytes ([kv_head][page_size][head_dim/64] fp16): the vector engine moves them
    through a random per-page table; the TMA engine refuses granules below 1 KiB up front."""
    torch = torch_cuda
    pb, pages = 64, 3000
    rng = np.random.default_rng(3)
    host_src = rng.integers(0, 256, pages * pb, dtype=np.uint8)
    table = O.permutation(4096, seed=8)[:pages]
    src = torch.from_numpy(host_src).cuda()
    pool = torch.zeros(4096 * pb, dtype=torch.uint8, device="cuda")
    dt = torch.from_numpy(table.copy()).cuda()
    seg = skv.segment(src, pool, pages * pb, dst_pages=dt, page_bytes=pb, dst_page_limit=4096)
    assert run(torch, [seg], skv.COPY_AUTO) == 0
    expect = np.zeros(4096 * pb, dtype=np.uint8)
    O.scatter_pages(host_src, table, pages, pb, expect)
    assert (pool.cpu().numpy() == expect).all()
    with pytest.raises(skv.SkvError, match="TMA engine"):
        skv.copy([seg], skv.COPY_TMA)


def test_empty_and_refused_segments(torch_cuda):
    torch = torch_cuda
    a = torch.zeros(64, dtype=torch.uint8, device="cuda")
    skv.copy([skv.segment(a, a, 0)], skv.COPY_TMA)          # zero bytes: nothing launched
    with pytest.raises(skv.SkvError, match="16-byte aligned"):
        skv.copy([skv.segment(a.data_ptr() + 8, a, 16)], skv.COPY_VEC)
    with pytest.raises(skv.SkvError, match="page_bytes"):
        skv.copy([skv.segment(a, a, 48, dst_pages=a, page_bytes=32, dst_page_limit=1)], skv.COPY_VEC)
    torch.cuda.synchronize()


def test_flag_wait_times_out_and_signal_releases(torch_cuda):
    """A wait on a flag nobody sets ends by itself after its limit with the timeout bit set (the context
    stays usable); a signal after a copy releases a second wait immediately."""
    torch = torch_cuda
    flag = torch.zeros(2, dtype=torch.int64, device="cuda")
    skv.clear_status(0)
    skv.lib().skv_wait_flag(flag.data_ptr(), 1, 50_000_000, None)
    torch.cuda.synchronize()
    assert skv.query_status(0) == skv.STATUS_WAIT_TIMEOUT
    skv.clear_status(0)
    src = torch.arange(1024, dtype=torch.int32, device="cuda")
    dst = torch.zeros_like(src)
    skv.copy([skv.segment(src, dst, 4096)], skv.COPY_VEC)
    skv.check(skv.lib().skv_signal(flag.data_ptr(), 7, None))
    skv.check(skv.lib().skv_wait_flag(flag.data_ptr(), 7, 1_000_000_000, None))
    torch.cuda.synchronize()
    assert skv.query_status(0) == 0 and torch.equal(src, dst) and int(flag[0]) == 7


def test_gated_copy_waits_releases_and_times_out(torch_cuda):
    """skv_copy_gated on one GPU.  A gate raised earlier on the same stream opens the copy, which lands exactly the
    oracle's scatter and then raises its done flag; a gate nobody raises ends after its limit with the timeout bit,
    nothing moved and no done flag; done-only launches twice in a row each raise their flag (the shared counters
    start from zero again after every launch, the timed-out one included)."""
    torch = torch_cuda
    pb, pages, limit = 4096, 200, 512
    image = np.random.default_rng(5).integers(0, 256, pages * pb, dtype=np.uint8)
    table = O.permutation(limit, seed=6)[:pages].copy()
    expect = np.full(limit * pb, 0x77, dtype=np.uint8)
    O.scatter_pages(image, table, pages, pb, expect)
    src = torch.from_numpy(image).cuda()
    pool = torch.full((limit * pb,), 0x77, dtype=torch.uint8, device="cuda")
    dt = torch.from_numpy(table).cuda()
    flags = torch.zeros(4, dtype=torch.int64, device="cuda")
    f = [flags.data_ptr() + 8 * i for i in range(4)]
    seg = skv.segment(src, pool, pages * pb, dst_pages=dt, page_bytes=pb, dst_page_limit=limit)
    skv.clear_status(0)
    skv.signal(f[0], 3)                                     # the gate, raised before the copy on the same stream
    skv.copy_gated([seg], f[0], 3, f[1], 9, timeout_ns=1_000_000_000)
    torch.cuda.synchronize()
    assert skv.query_status(0) == 0 and int(flags[1]) == 9
    assert (pool.cpu().numpy() == expect).all()

    pool.fill_(0x77)
    skv.clear_status(0)
    skv.copy_gated([seg], f[2], 1, f[3], 5, timeout_ns=2_000_000)   # nobody raises f[2]
    torch.cuda.synchronize()
    assert skv.query_status(0) == skv.STATUS_WAIT_TIMEOUT
    assert int(flags[3]) == 0 and int((pool != 0x77).sum()) == 0

    skv.clear_status(0)
    for v in (11, 12):
        skv.copy_gated([seg], None, 0, f[3], v)
        torch.cuda.synchronize()
        assert int(flags[3]) == v
    assert skv.query_status(0) == 0 and (pool.cpu().numpy() == expect).all()
    with pytest.raises(skv.SkvError, match="nothing to move"):
        skv.copy_gated([skv.segment(src, pool, 0)], None, 0, f[3], 1)
