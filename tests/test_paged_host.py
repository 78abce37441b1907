"""Host-side page allocator of PagedBatchCache (no GPU: tensors on the CPU,
nothing calls the library)."""
from __future__ import annotations

import pytest

import eckv


def _cache(**kw):
    return eckv.PagedBatchCache(3, num_pages=6, page_tokens=128, device="cpu", **kw)


def test_reserve_grows_page_by_page_and_fills_the_row():
    c = _cache()
    c.reserve(0, 1)
    assert c.pages[0] == [0] and int(c.capacity[0]) == 128
    c.reserve(0, 128)                       # still one page
    assert c.pages[0] == [0]
    c.reserve(0, 129)
    assert c.pages[0] == [0, 1] and int(c.capacity[0]) == 256
    assert c.page_table[0].tolist() == [0, 1, -1, -1, -1, -1]
    assert c.slot(0, 130) == 1 * 128 + 2


def test_sequences_draw_disjoint_pages_and_exhaustion_raises():
    c = _cache(shuffle_seed=3)
    c.reserve(0, 300)
    c.reserve(1, 300)
    assert not set(c.pages[0]) & set(c.pages[1])
    with pytest.raises(MemoryError):
        c.reserve(2, 128 * 3)               # 6 pages, 6 already asked for
    with pytest.raises(ValueError):
        c.reserve(2, 128 * 7)               # past max_pages


def test_release_returns_pages_for_reuse():
    c = _cache()
    c.reserve(0, 600)                       # 5 pages
    c.length[0] = 600
    taken = list(c.pages[0])
    c.release(0)
    assert c.pages[0] == [] and int(c.capacity[0]) == 0 and int(c.length[0]) == 0
    assert c.page_table[0].tolist() == [-1] * 6
    c.reserve(1, 128 * 6)                   # the whole pool again
    assert sorted(c.pages[1]) == sorted(taken + [5])


def test_page_size_must_be_a_power_of_two_of_at_least_128():
    with pytest.raises(ValueError):
        eckv.PagedBatchCache(1, num_pages=2, page_tokens=192, device="cpu")
    with pytest.raises(ValueError):
        eckv.PagedBatchCache(1, num_pages=2, page_tokens=64, device="cpu")
