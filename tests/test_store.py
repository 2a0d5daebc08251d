"""The host parity store's ring (CPU; unpinned memory)."""
from __future__ import annotations

import random

import pytest

from conftest import pkg


def make(keep=256, budget=1 << 20):
    released = []
    st = pkg("store").ParityStore(keep, budget, pin=False, before_release=lambda: released.append(1))
    return st, released


def fill(entry, tag):
    entry["host"].fill_(tag % 251 + 1)


def intact(entry, tag):
    return bool((entry["host"] == tag % 251 + 1).all())


def test_equal_chunks_wrap_and_drop_the_oldest():
    st, _ = make(keep=256, budget=4096)  # room for 4 chunks of 1 KiB
    for cid in range(1, 7):
        fill(st.put(cid, 1024), cid)
    assert st.keys() == [3, 4, 5, 6]
    assert st.block_bytes == 4096
    assert all(intact(st[c], c) for c in st.keys())


def test_count_limit():
    st, _ = make(keep=3, budget=1 << 20)
    for cid in range(1, 6):
        st.put(cid, 100)
    assert st.keys() == [3, 4, 5]


def test_same_chunk_again_reuses_its_bytes():
    st, _ = make(keep=256, budget=4096)
    for cid in range(1, 5):
        fill(st.put(cid, 1024), cid)
    off = st[4]["off"]
    fill(st.put(4, 1024), 40)
    assert st[4]["off"] == off and st.keys() == [1, 2, 3, 4]
    assert intact(st[4], 40) and all(intact(st[c], c) for c in (1, 2, 3))


def test_larger_chunk_takes_a_new_block_and_keeps_the_old_chunks_readable():
    st, released = make(keep=256, budget=4096)
    for cid in range(1, 4):
        fill(st.put(cid, 1024), cid)
    fill(st.put(4, 8192), 4)  # does not fit: a larger block
    assert released == [1]
    assert st.block_bytes >= 4 * 8192
    assert st.keys() == [1, 2, 3, 4]
    assert all(intact(st[c], c) for c in st.keys())


def test_missing_chunk():
    st, _ = make()
    assert st.get(7) is None and 7 not in st
    with pytest.raises(KeyError):
        st[7]


@pytest.mark.parametrize("seed", range(20))
def test_random_sizes_never_corrupt_a_kept_chunk(seed):
    rnd = random.Random(seed)
    st, _ = make(keep=rnd.choice([4, 16, 256]), budget=rnd.choice([4096, 20000, 1 << 16]))
    tags = {}
    for step in range(300):
        cid = rnd.randrange(1, 60) if rnd.random() < 0.3 else 1000 + step  # some ids stored again
        n = rnd.choice([16, 48, 512, 1024, 3000, 5000]) if rnd.random() < 0.97 else 70000
        e = st.put(cid, n)
        tags[cid] = step
        fill(e, step)
        assert len(st) <= st.keep
        for c in st.keys():  # every chunk still kept holds exactly what was written
            assert intact(st[c], tags[c]), (seed, step, c)
        live = sorted((st[c]["off"], st[c]["off"] + st[c]["size"]) for c in st.keys()
                      if st[c]["gen"] == st[cid]["gen"])
        assert all(a[1] <= b[0] for a, b in zip(live, live[1:]))  # no two kept chunks share bytes
