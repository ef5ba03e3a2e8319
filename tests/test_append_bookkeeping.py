"""The host side of a decode append (``HeteroCache._append_bookkeeping``:
the free-list check of heterocache/cache_utils.py:981-990 on the mirrored
lengths) with its slack fast path, against the plain per-append check
restated below: the same lengths, mapped pages, free-list pointer and the
same exception at the same append, over random ragged states, including
rows that start on a page boundary, rows without pages and tables that run
out of columns.  No GPU."""
import types

import numpy as np
import pytest
import torch

from heterocache_b200.cache import HeteroCache

PAGE = 256


def _plain(st):
    """One append, checked in full (the bookkeeping without its fast path)."""
    hl, mapped = st["hlen"], st["mapped"]
    logical = hl // PAGE
    if np.any(logical >= st["width"]):
        raise IndexError("no column")
    grow = logical >= mapped
    need = int(np.count_nonzero(grow))
    if need:
        if st["ptr"] + need > st["free"]:
            raise RuntimeError("OOM")
        st["ptr"] += need
        mapped += grow
    hl += 1


def _cache(hl, mapped, width, free):
    c = types.SimpleNamespace(_hlen=[hl.copy()], _mapped=[mapped.copy()], _slack=[0],
                              block_tables=[torch.zeros(len(hl), width, dtype=torch.int32)],
                              free_blocks=[torch.zeros(free, dtype=torch.int32)], free_block_pointers=[0])
    return c


@pytest.mark.parametrize("seed", range(12))
def test_slack_path_matches_the_full_check(seed):
    rng = np.random.default_rng(seed)
    rows = int(rng.integers(1, 9))
    width = int(rng.integers(2, 12))
    hl = rng.integers(0, 3 * PAGE, rows).astype(np.int64)
    if seed % 3 == 0:
        hl[0] = PAGE * int(rng.integers(0, 3))  # on a page boundary
    mapped = np.minimum((hl + PAGE - 1) // PAGE + rng.integers(0, 2, rows), width).astype(np.int64)
    if seed % 4 == 1:
        mapped[-1] = 0
        hl[-1] = 0  # a row without pages
    free = int(rng.integers(0, 3 * rows + 2))
    ref = {"hlen": hl.copy(), "mapped": mapped.copy(), "ptr": 0, "free": free, "width": width}
    c = _cache(hl, mapped, width, free)
    for step in range(width * PAGE + 10):
        want = None
        try:
            _plain(ref)
        except (IndexError, RuntimeError) as e:
            want = type(e)
        if want is not None:
            with pytest.raises(want):
                HeteroCache._append_bookkeeping(c, 0)
            return
        HeteroCache._append_bookkeeping(c, 0)
        assert np.array_equal(c._hlen[0], ref["hlen"]), step
        assert np.array_equal(c._mapped[0], ref["mapped"]), step
        assert c.free_block_pointers[0] == ref["ptr"], step
    pytest.fail("no append ran out of columns")


def test_slack_skips_the_checks_between_page_edges():
    c = _cache(np.array([10, 300], dtype=np.int64), np.array([1, 2], dtype=np.int64), 8, 4)
    HeteroCache._append_bookkeeping(c, 0)
    assert c._slack[0] == min(256 - 11, 512 - 301)
    for _ in range(c._slack[0]):
        HeteroCache._append_bookkeeping(c, 0)
    assert c._slack[0] == 0 and c._hlen[0].tolist() == [222, 512]
    HeteroCache._append_bookkeeping(c, 0)  # row 1 crosses into a new page first
    assert c._mapped[0].tolist() == [1, 3] and c.free_block_pointers[0] == 1
    assert c._slack[0] == 256 - 223
