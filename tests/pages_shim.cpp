// C entry points over hyk::PagePool (hymt2_b200/csrc/hy_pages.h) for the CPU
// tests of the paged KV cache's host logic; compiled by tests/test_pages.py.
#include "../hymt2_b200/csrc/hy_pages.h"

using hyk::PagePool;

extern "C" {
void *hp_create(int npages) {
    PagePool *p = new PagePool();
    p->reset(npages);
    return p;
}
void hp_destroy(void *h) { delete (PagePool *)h; }
int hp_alloc(void *h) { return ((PagePool *)h)->alloc(); }
void hp_ref(void *h, int p) { ((PagePool *)h)->ref(p); }
void hp_unref(void *h, int p) { ((PagePool *)h)->unref(p); }
int hp_seal(void *h, int p, int parent, const int *toks) { return ((PagePool *)h)->seal(p, parent, toks) ? 1 : 0; }
// rows matched; full pages into full[0 .. cap), their count into *nfull
int hp_match(void *h, const int *toks, int limit, int *full, int cap, int *nfull, int *src, int *src_rows) {
    PagePool::Match m = ((PagePool *)h)->match(toks, limit);
    int n = 0;
    for (int p : m.full)
        if (n < cap) full[n++] = p;
    *nfull = (int)m.full.size();
    *src = m.src;
    *src_rows = m.src_rows;
    return m.rows;
}
int hp_free_count(void *h) { return ((PagePool *)h)->free_count(); }
int hp_cached_idle(void *h) { return ((PagePool *)h)->cached_idle(); }
long long hp_evictions(void *h) { return ((PagePool *)h)->evictions(); }
int hp_refs(void *h, int p) { return ((PagePool *)h)->refs(p); }
int hp_cached(void *h, int p) { return ((PagePool *)h)->cached(p) ? 1 : 0; }
int hp_page_rows(void) { return hyk::kPageRows; }
}
