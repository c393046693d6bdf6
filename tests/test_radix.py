"""The page-granular prefix cache (msgl_radix_*, host side, no GPU) against a brute-force model.

The model keeps one entry per cached page, keyed by the whole token prefix that ends with that
page: a match is the longest run of cached prefixes, insert adds the missing ones, a lock counts
on every page of a path, and eviction removes the least recently used unlocked page that no
other page extends (ties: the lower page id). The tree must give the same matches, duplicate
pages, freed pages and sizes over random operation sequences, plus the reference's own radix
test (tests/unit/test_scheduler.cpp:24-40) at page size 1.
"""
import numpy as np
import pytest

from msgl.model import RadixCache


class PageModel:
    def __init__(self, P):
        self.P, self.e, self.clock = P, {}, 0  # e: prefix tuple -> [page, time, ref]

    def _walk(self, t, n):
        keys = []
        while (len(keys) + 1) * self.P <= n and tuple(t[:(len(keys) + 1) * self.P]) in self.e:
            keys.append(tuple(t[:(len(keys) + 1) * self.P]))
        return keys

    def _touch(self, keys):
        self.clock += 1
        for k in keys:
            self.e[k][1] = self.clock

    def match(self, t):
        keys = self._walk(t, len(t))
        self._touch(keys)
        return len(keys) * self.P, [self.e[k][0] for k in keys], (keys[-1] if keys else ())

    def insert(self, t, pages):
        full = len(t) - len(t) % self.P
        keys = self._walk(t, full)
        dup = [pages[i] for i, k in enumerate(keys) if pages[i] != self.e[k][0]]
        present = len(keys) * self.P
        for j in range(len(keys), full // self.P):
            k = tuple(t[:(j + 1) * self.P])
            self.e[k] = [pages[j], 0, 0]
            keys.append(k)
        self._touch(keys)
        return present, dup, (keys[-1] if keys else ())

    def lock(self, key, d):
        for j in range(1, len(key) // self.P + 1):
            self.e[key[:j * self.P]][2] += d

    def evict(self, n):
        freed = []
        while len(freed) < n:
            inner = {k[:-self.P] for k in self.e if len(k) > self.P}
            leaves = [k for k in self.e if k not in inner and self.e[k][2] == 0]
            if not leaves:
                break
            k = min(leaves, key=lambda k: (self.e[k][1], self.e[k][0]))
            freed.append(self.e.pop(k)[0])
        return freed

    def size(self):
        return len(self.e), sum(1 for v in self.e.values() if v[2] == 0)


def test_reference_radix_test_at_page_size_one():
    r = RadixCache(page_size=1)
    r.insert([1, 2, 3, 4, 5], [10, 11, 12, 13, 14])
    m, pages, _ = r.match([1, 2, 3, 4, 5])
    assert m == 5 and pages == [10, 11, 12, 13, 14]
    m, pages, _ = r.match([1, 2, 3, 9, 10])
    assert m == 3 and pages == [10, 11, 12]


def test_siblings_split_and_partial_pages():
    r = RadixCache(page_size=4)
    a = [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12]
    b = [1, 2, 3, 4, 5, 6, 7, 99, 0, 0, 0, 0]  # diverges inside the second page
    assert r.insert(a, [100, 101, 102])[0] == 0
    present, dup, _ = r.insert(b, [100, 201, 202])  # shares only the first page
    assert present == 4 and dup == []
    assert r.match(a) == (12, [100, 101, 102], r.match(a)[2])
    assert r.match(b)[:2] == (12, [100, 201, 202])
    assert r.match(a[:7])[:2] == (4, [100])  # a partial page never matches
    present, dup, _ = r.insert(a + [13, 14], [300, 301, 302, 303])  # same prefix, other pages
    assert present == 12 and dup == [300, 301, 302]  # the caller frees its copies
    assert r.size() == (5, 5)


def test_locked_paths_are_not_evicted():
    r = RadixCache(page_size=2)
    _, _, n1 = r.insert([1, 1, 2, 2, 3, 3], [1, 2, 3])
    _, _, n2 = r.insert([1, 1, 5, 5], [1, 9])
    r.lock(n1)
    assert r.evict(10) == [9]  # only the unlocked leaf goes
    assert r.size() == (3, 0)
    r.lock(n1, -1)
    assert r.evict(10) == [3, 2, 1]
    assert r.size() == (0, 0)
    with pytest.raises(Exception):
        r.lock(n2)  # evicted node: stale handle


@pytest.mark.parametrize("seed,P", [(0, 1), (1, 2), (2, 4), (3, 2), (4, 3)])
def test_random_operations_match_the_page_model(seed, P):
    rng = np.random.default_rng(seed)
    tree, model = RadixCache(page_size=P), PageModel(P)
    handles = []   # (tree node id, model key) of recent matches / inserts
    locked = []
    next_page = 1000
    for step in range(1500):
        op = rng.integers(0, 10)
        seq = [int(x) for x in rng.integers(0, 3, rng.integers(0, 18))]
        if op < 3:
            got, want = tree.match(seq), model.match(seq)
            assert got[:2] == want[:2], (step, seq)
            handles.append((got[2], want[2]))
        elif op < 6:
            n = len(seq) // P
            cached = []
            if rng.integers(0, 2):  # a scheduler matches first and reuses the cached pages
                got, want = tree.match(seq), model.match(seq)
                assert got[:2] == want[:2], (step, seq)
                cached = want[1]
            pages = cached + list(range(next_page, next_page + n - len(cached)))
            if rng.integers(0, 3) == 0:  # sometimes fresh pages for the cached part too
                pages = list(range(next_page, next_page + n))
            next_page += n
            got, want = tree.insert(seq, pages), model.insert(seq, pages)
            assert got[:2] == want[:2], (step, seq)
            handles.append((got[2], want[2]))
        elif op == 6 and handles:
            h = handles[rng.integers(0, len(handles))]
            if h[1] in model.e or h[1] == ():
                tree.lock(h[0], 1)
                model.lock(h[1], 1)
                locked.append(h)
        elif op == 7 and locked:
            h = locked.pop(rng.integers(0, len(locked)))
            tree.lock(h[0], -1)
            model.lock(h[1], -1)
        elif op == 8:
            k = int(rng.integers(0, 6))
            assert tree.evict(k) == model.evict(k), step
            handles = [h for h in handles if h in locked or h[1] == () or h[1] in model.e]
        assert tree.size() == model.size(), step
