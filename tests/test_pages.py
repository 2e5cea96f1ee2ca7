"""Host logic of the paged KV cache (hymt2_b200/csrc/hy_pages.h), on the CPU.

The page pool and shared-prefix page cache that the continuous-batching
server (hy_batch.cuh serve_run) drives, through a small C shim compiled
here.  Besides unit cases (chain sharing, the copied tail, LRU eviction,
stale children, reference counts) a randomised server simulation checks the
property the GPU server relies on: every KV row a sequence reads through its
page table was written for exactly its own token prefix (a row at position i
depends on tokens 0..i), whichever request wrote it and however pages were
shared, copied, evicted and reused.  Reference semantics: longest-common-
prefix reuse of src/model.c:931-936, across every cached prompt.
"""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
R = 16


@pytest.fixture(scope="module")
def hp(tmp_path_factory):
    so = str(tmp_path_factory.mktemp("pages") / "libhypages.so")
    subprocess.run(["g++", "-O1", "-std=c++17", "-shared", "-fPIC", "-o", so, os.path.join(HERE, "pages_shim.cpp")],
                   check=True)
    L = C.CDLL(so)
    P, I = C.c_void_p, C.c_int
    L.hp_create.restype = P
    L.hp_create.argtypes = [I]
    for f in ("hp_destroy",):
        getattr(L, f).argtypes = [P]
    for f in ("hp_alloc", "hp_free_count", "hp_cached_idle"):
        getattr(L, f).argtypes = [P]
        getattr(L, f).restype = I
    L.hp_evictions.argtypes = [P]
    L.hp_evictions.restype = C.c_longlong
    for f in ("hp_ref", "hp_unref"):
        getattr(L, f).argtypes = [P, I]
    for f in ("hp_refs", "hp_cached"):
        getattr(L, f).argtypes = [P, I]
        getattr(L, f).restype = I
    L.hp_seal.argtypes = [P, I, I, P]
    L.hp_seal.restype = I
    L.hp_match.argtypes = [P, P, I, P, I, P, P, P]
    L.hp_match.restype = I
    assert L.hp_page_rows() == R
    return L


class Pool:
    def __init__(self, L, n):
        self.L, self.h = L, L.hp_create(n)

    def alloc(self):
        return self.L.hp_alloc(self.h)

    def ref(self, p):
        self.L.hp_ref(self.h, p)

    def unref(self, p):
        self.L.hp_unref(self.h, p)

    def seal(self, p, parent, toks):
        a = np.ascontiguousarray(toks, dtype=np.int32)
        return bool(self.L.hp_seal(self.h, p, parent, a.ctypes.data))

    def match(self, toks, limit):
        a = np.ascontiguousarray(toks, dtype=np.int32)
        full = np.zeros(256, dtype=np.int32)
        nf, src, sr = C.c_int(), C.c_int(), C.c_int()
        rows = self.L.hp_match(self.h, a.ctypes.data, limit, full.ctypes.data, 256, C.byref(nf), C.byref(src),
                               C.byref(sr))
        return rows, full[:nf.value].tolist(), src.value, sr.value

    def free_count(self):
        return self.L.hp_free_count(self.h)

    def idle(self):
        return self.L.hp_cached_idle(self.h)

    def evictions(self):
        return self.L.hp_evictions(self.h)

    def close(self):
        self.L.hp_destroy(self.h)


def _fill(pool, toks):
    """A fed prompt: one page per 16 rows, its full pages sealed in a chain."""
    pages = [pool.alloc() for _ in range((len(toks) + R - 1) // R)]
    for j in range(len(toks) // R):
        pool.seal(pages[j], pages[j - 1] if j else -1, toks[j * R:(j + 1) * R])
    return pages


def test_chain_share_and_copied_tail(hp):
    pool = Pool(hp, 32)
    try:
        rng = np.random.default_rng(1)
        a = rng.integers(0, 1000, 50).tolist()          # 3 full pages + 2 rows
        pa = _fill(pool, a)
        b = a[:40] + rng.integers(0, 1000, 10).tolist()  # shares 2 pages + 8 rows of page 2
        rows, full, src, sr = pool.match(b, len(b) - 1)
        assert rows == 40 and full == pa[:2] and src == pa[2] and sr == 8
        assert hp.hp_refs(pool.h, pa[0]) == 2 and hp.hp_refs(pool.h, pa[2]) == 1   # match references full pages only
        # the last prompt token is never reused: limit n - 1
        rows, full, src, sr = pool.match(a[:32], 31)
        assert rows == 31 and full == pa[:1] and src == pa[1] and sr == 15
        # a prompt shorter than a page reuses rows of a cached first page
        rows, full, src, sr = pool.match(a[:9], 8)
        assert rows == 8 and full == [] and src == pa[0] and sr == 8
        # different first token: nothing
        assert pool.match([a[0] + 1] + a[1:], 49)[0] == 0
    finally:
        pool.close()


def test_equal_pages_stay_private_and_refs_free(hp):
    pool = Pool(hp, 8)
    try:
        t = list(range(100, 132))
        p1 = _fill(pool, t)
        p2 = [pool.alloc(), pool.alloc()]
        assert not pool.seal(p2[0], -1, t[:16])          # an equal page is cached
        assert pool.free_count() == 4
        for p in p2:
            pool.unref(p)                                # private: back to the free list
        assert pool.free_count() == 6
        for p in p1:
            pool.unref(p)                                # cached: idle, not free
        assert pool.free_count() == 6 and pool.idle() == 2
        rows, full, _, _ = pool.match(t + [7], 32)
        assert rows == 32 and full == p1 and pool.idle() == 0
    finally:
        pool.close()


def test_lru_eviction_and_unreachable_children(hp):
    pool = Pool(hp, 4)
    try:
        a = list(range(0, 32))
        b = list(range(500, 532))
        pa = _fill(pool, a)
        pb = _fill(pool, b)
        for p in pa + pb:
            pool.unref(p)
        assert pool.free_count() == 0 and pool.idle() == 4
        # touch b's chain (match references, then release): a's pages are now the oldest
        _, fb, _, _ = pool.match(b + [1], 32)
        for p in fb:
            pool.unref(p)
        x = pool.alloc()
        assert x == pa[0] and pool.evictions() == 1      # a's first page went first
        # a's second page is unreachable without its parent, and a new equal
        # first page replaces the stale entry of the child on sealing
        assert pool.match(a + [1], 32)[0] == 0
        pool.unref(x)
        p0 = pool.alloc()
        assert pool.seal(p0, -1, a[:16])
        rows, full, src, sr = pool.match(a + [1], 32)
        assert full == [p0] and rows == 16 + sr and src in (-1, pa[1])
        # every page referenced: no page to give
        keep = [pool.alloc() for _ in range(pool.free_count() + pool.idle())]
        assert pool.alloc() == -1
        for p in keep:
            pool.unref(p)
    finally:
        pool.close()


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_server_simulation_rows_match_their_prefix(hp, seed):
    """serve_run's page bookkeeping on random requests (shared prefixes of
    random length, slots fewer than requests, a pool that forces evictions):
    every row a sequence reads was written for its own token prefix."""
    rng = np.random.default_rng(seed)
    slots, slot_ctx = 4, 96
    page_max = slot_ctx // R
    npages = slots * page_max + max(page_max, slots * page_max // 4)
    pool = Pool(hp, npages)
    content = {}                                    # (page, row) -> token prefix that produced it
    stems = [rng.integers(0, 50, int(rng.integers(8, 60))).tolist() for _ in range(5)]
    reqs = []
    for _ in range(60):
        s = stems[int(rng.integers(0, len(stems)))]
        cut = int(rng.integers(1, len(s) + 1))
        reqs.append(s[:cut] + rng.integers(0, 50, int(rng.integers(1, 20))).tolist())
    max_new, hits, shared = 5, 0, 0
    active, nxt, done = [], 0, 0
    try:
        while done < len(reqs):
            while len(active) < slots and nxt < len(reqs):
                toks = reqs[nxt]
                n = len(toks)
                rows, full, src, sr = pool.match(toks, n - 1)
                q = {"toks": list(toks), "n": n, "pages": list(full), "fed": rows, "gen": 0, "sealed": False}
                if src >= 0 and sr > 0:
                    pool.ref(src)
                    dst = pool.alloc()
                    assert dst >= 0
                    q["pages"].append(dst)
                    for i in range(sr):
                        content[(dst, i)] = content[(src, i)]
                    pool.unref(src)
                for i in range(rows):                       # what the sequence will read
                    assert content[(q["pages"][i // R], i % R)] == tuple(toks[:i + 1])
                hits += rows > 0
                shared += len(full)
                active.append(q)
                nxt += 1
            for q in active:                                # one step: a chunk or a decode token each
                if q["fed"] < q["n"]:
                    take = min(q["n"] - q["fed"], int(rng.integers(1, 40)))
                    pos = range(q["fed"], q["fed"] + take)
                    q["fed"] += take
                else:
                    pos = [q["n"] + q["gen"] - 1]
                    q["toks"].append(int(rng.integers(0, 50)))   # the generated id fed next
                    q["gen"] += 1
                for p in pos:
                    while len(q["pages"]) <= p // R:
                        pg = pool.alloc()
                        assert pg >= 0, "pool exhausted"
                        q["pages"].append(pg)
                    content[(q["pages"][p // R], p % R)] = tuple(q["toks"][:p + 1])
                    for i in range(p + 1):              # attention reads rows 0..p
                        assert content[(q["pages"][i // R], i % R)] == tuple(q["toks"][:i + 1])
            for q in active:                                # seal fed prompts
                if q["sealed"] or q["fed"] < q["n"]:
                    continue
                q["sealed"] = True
                for j in range(q["n"] // R):
                    pg = q["pages"][j]
                    if not hp.hp_cached(pool.h, pg) and not pool.seal(pg, q["pages"][j - 1] if j else -1,
                                                                        q["toks"][j * R:(j + 1) * R]):
                        break
            keep = []
            for q in active:
                if q["fed"] == q["n"] and q["gen"] >= max_new:
                    for pg in q["pages"]:
                        pool.unref(pg)
                    done += 1
                else:
                    keep.append(q)
            active = keep
        assert hits > 10 and shared > 5
        assert pool.evictions() > 0
        assert pool.free_count() + pool.idle() == npages   # every reference returned
    finally:
        pool.close()
