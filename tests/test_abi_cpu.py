"""The C ABI without a GPU: the library loads, exports every symbol include/strata_kv.h declares, and its
host-side logic (the block allocator, table expansion, argument refusals) behaves.  No kernel is launched."""
import os
import re
import subprocess

import numpy as np
import pytest

import oracle as O
import skv

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "strata_kv.h")


def declared_symbols(path):
    text = open(path).read()
    return sorted(set(re.findall(r"^SKV_API [^;(]*?\b(skv_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = skv.lib()
    names = declared_symbols(HEADER)
    assert len(names) >= 25
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", skv.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (skv_\w+)", out))
    assert set(names) <= exported
    assert set(skv.exported_names()) == set(names), "the Python binding covers exactly the header"
    assert lib.skv_version() == 1


def fake_pool(n_blocks=16, block_bytes=4096):
    # a wrapped pool is host bookkeeping only; the base address is never dereferenced here
    return skv.Pool(0, n_blocks, block_bytes, memory=0x10000)


def test_allocator_all_or_nothing_and_double_free():
    p = fake_pool(8)
    a = p.alloc(5)
    assert sorted(a.tolist()) == [0, 1, 2, 3, 4] and p.free_count() == 3
    with pytest.raises(skv.SkvError) as e:
        p.alloc(4)
    assert e.value.code == skv.ENOMEM and p.free_count() == 3
    p.free(a[:2])
    with pytest.raises(skv.SkvError, match="not allocated"):
        p.free(a[:1])                     # double free refused
    with pytest.raises(skv.SkvError, match="listed twice"):
        p.free([a[2], a[2]])
    assert p.free_count() == 5            # the refused frees freed nothing
    with pytest.raises(skv.SkvError):
        p.free([99])
    p.close()


def test_allocator_scramble_is_seeded():
    def order(seed):
        p = fake_pool(64)
        p.scramble(seed)
        out = p.alloc(64).tolist()
        p.close()
        return out
    a, b, c = order(1), order(1), order(2)
    assert a == b and a != c and sorted(a) == list(range(64))


def test_expand_block_table_matches_oracle():
    blocks = O.permutation(40, seed=3)[:10]
    for off in (0, 64):
        assert (skv.expand_block_table(blocks, 64, 128, off) == O.expand_block_table(blocks, 64, 128, off)).all()
    with pytest.raises(skv.SkvError):
        skv.expand_block_table(blocks, 64, 64, 64)           # offset + pages past the slot
    with pytest.raises(skv.SkvError):
        skv.expand_block_table(np.array([2 ** 30], dtype=np.int32), 64, 128, 0)   # page index past int32


def test_pool_wrap_refuses_bad_arguments():
    with pytest.raises(skv.SkvError):
        skv.Pool(0, 0, 4096, memory=0x10000)
    with pytest.raises(skv.SkvError):
        skv.Pool(0, 4, 4096, memory=0x10001)                 # misaligned base
    with pytest.raises(skv.SkvError):
        skv.Pool(0, 4, 1000, memory=0x10000)                 # slot not a multiple of 1 KiB


def test_geometry_and_metric_bytes():
    g = skv.KvGeometry()
    assert g.page_bytes == 4096 and g.block_bytes == 512 * 1024
    assert g.gdn_bytes == 79036416
    assert g.metric_bytes(32768) == 24576 * 32768 + 79036416 + 4 * 32768
    assert g.metric_bytes(4096) == O.metric_bytes(O.Geometry(), 4096)
    off = skv.image_offsets(g, 5, 2)
    assert off[(0, 1)] == 2 * 4096 and off["total"] % 256 == 0


def test_allocator_under_threads_never_hands_out_a_held_block():
    """Eight threads allocate and free from one pool at once (the C calls release the GIL): a block is never
    handed to two holders, and every block is free again at the end."""
    import threading
    p = fake_pool(256)
    held, lock, errors = {}, threading.Lock(), []

    def worker(t):
        rng = np.random.default_rng(t)
        mine = []
        try:
            for _ in range(400):
                if mine and rng.random() < 0.5:
                    k = int(rng.integers(1, len(mine) + 1))
                    give, mine = mine[:k], mine[k:]
                    with lock:
                        for b in give:
                            del held[b]
                    p.free(give)
                else:
                    try:
                        got = p.alloc(int(rng.integers(1, 9))).tolist()
                    except skv.SkvError as e:
                        assert e.code == skv.ENOMEM
                        continue
                    with lock:
                        for b in got:
                            assert b not in held, f"block {b} handed to thread {t} while thread {held[b]} holds it"
                            held[b] = t
                    mine += got
            with lock:
                for b in mine:
                    del held[b]
            p.free(mine)
        except Exception as e:   # surfaced below: a failing thread must fail the test
            errors.append(e)

    threads = [threading.Thread(target=worker, args=(t,)) for t in range(8)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors[0]
    assert p.free_count() == 256 and not held
    p.close()


def test_gated_copy_refuses_bad_flags_before_touching_a_device():
    """skv_copy_gated checks its flags and its timeout before anything reaches a device."""
    seg = (skv.Segment * 1)(skv.segment(0x1000, 0x2000, 4096))
    L = skv.lib()
    assert L.skv_copy_gated(seg, 1, 0x1004, 1, 0, None, 0, None) == skv.EINVAL          # misaligned wait flag
    assert "8-byte aligned" in L.skv_last_error().decode()
    assert L.skv_copy_gated(seg, 1, None, 0, 0, 0x2002, 1, None) == skv.EINVAL          # misaligned done flag
    assert L.skv_copy_gated(seg, 1, 0x1000, 1, 61 * 10 ** 9, None, 0, None) == skv.EINVAL   # timeout past 60 s
    assert "60 s" in L.skv_last_error().decode()
