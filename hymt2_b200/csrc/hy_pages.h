// hy_pages.h — host side of the paged KV cache: which device page holds
// which rows, and the shared-prefix page cache of the continuous-batching
// server.  Plain C++ (no CUDA): the server owns the device pages and copies;
// this class only decides.
//
// A page holds kPageRows consecutive positions of one sequence in every
// layer.  A request's prompt rows depend only on its prompt tokens, so once
// a prompt is fed, each of its full pages is immutable and can serve every
// later prompt that starts with the same tokens: the page is sealed into
// the cache under a chain hash of all tokens up to its last row (page j's
// key covers tokens 0 .. 16 j + 15) and shared by reference, with no copy.
// A new prompt reuses the longest chain of cached full pages that matches
// its tokens, then the first rows of one cached child page of the last
// match (copied into a page of its own), which generalises the reference's
// longest-common-prefix reuse against the previous prompt
// (src/model.c:931-936) to every cached prompt.  Pages nobody references
// stay cached in least-recently-used order and are evicted only when the
// free list is empty.
#pragma once
#include <cstdint>
#include <list>
#include <unordered_map>
#include <vector>

namespace hyk {

constexpr int kPageRows = 16;
constexpr int kPageShift = 4;
static_assert((1 << kPageShift) == kPageRows, "page rows must be a power of two");

class PagePool {
  public:
    struct Match {
        std::vector<int> full;  // shared full pages, referenced for the caller
        int src = -1;           // cached page whose first src_rows rows continue the match
        int src_rows = 0;
        int rows = 0;           // 16 * full.size() + src_rows
    };

    void reset(int npages) {
        pg_.assign((size_t)npages, Page());
        free_.clear();
        for (int p = npages - 1; p >= 0; p--) free_.push_back(p);
        lru_.clear();
        by_key_.clear();
        children_.clear();
        evictions_ = 0;
    }
    int pages() const { return (int)pg_.size(); }
    int free_count() const { return (int)free_.size(); }
    int cached_idle() const { return (int)lru_.size(); }
    long long evictions() const { return evictions_; }
    int refs(int p) const { return pg_[(size_t)p].ref; }
    bool cached(int p) const { return pg_[(size_t)p].cached; }

    // A page for new rows (referenced once), evicting the least recently
    // used idle cached page when no page is free; -1 when every page is
    // referenced.
    int alloc() {
        int p;
        if (!free_.empty()) {
            p = free_.back();
            free_.pop_back();
        } else if (!lru_.empty()) {
            p = lru_.front();
            evict(p);
        } else {
            return -1;
        }
        Page &g = pg_[(size_t)p];
        g.ref = 1;
        g.cached = false;
        g.in_lru = false;
        return p;
    }

    void ref(int p) {
        Page &g = pg_[(size_t)p];
        if (g.ref == 0 && g.in_lru) {
            lru_.erase(g.lru);
            g.in_lru = false;
        }
        g.ref++;
    }

    // Drop one reference; an unreferenced cached page waits in the LRU list,
    // any other goes back to the free list.
    void unref(int p) {
        Page &g = pg_[(size_t)p];
        if (g.ref <= 0) return;
        if (--g.ref > 0) return;
        if (g.cached) {
            g.lru = lru_.insert(lru_.end(), p);
            g.in_lru = true;
        } else {
            g.gen++;
            free_.push_back(p);
        }
    }

    // Seal full page p (its 16 rows are positions 16 j .. 16 j + 15 of a
    // prompt whose page j - 1 is `parent`, -1 for j = 0) holding the rows of
    // tokens toks[0 .. 16).  Returns false (p stays private) when an equal
    // page is cached already or the parent is not cached.
    bool seal(int p, int parent, const int *toks) {
        uint64_t pkey = kRootKey;
        uint32_t pgen = 0;
        if (parent >= 0) {
            const Page &q = pg_[(size_t)parent];
            if (!q.cached) return false;
            pkey = q.key;
            pgen = q.gen;
        }
        const uint64_t key = chain(pkey, toks);
        auto it = by_key_.find(key);
        if (it != by_key_.end()) {
            const Page &e = pg_[(size_t)it->second];
            if (e.parent == parent && e.parent_gen == pgen) return false;  // an equal page is cached
            unregister(it->second);  // a page whose parent was evicted: unreachable, replace it
        }
        Page &g = pg_[(size_t)p];
        if (g.cached) return false;
        g.cached = true;
        g.key = key;
        g.parent = parent;
        g.parent_gen = pgen;
        for (int i = 0; i < kPageRows; i++) g.toks[i] = toks[i];
        by_key_[key] = p;
        children_[child_key(parent, pgen)].push_back(p);
        return true;
    }

    // Longest cached prefix of toks[0 .. limit): full pages by chain hash
    // (each verified token for token and referenced for the caller), then
    // the cached child of the last one whose first rows match the most of
    // what follows.  The caller copies src's first src_rows rows before its
    // next alloc() could evict src.
    Match match(const int *toks, int limit) {
        Match m;
        int parent = -1;
        uint32_t pgen = 0;
        uint64_t key = kRootKey;
        int l = 0;
        while (l + kPageRows <= limit) {
            const uint64_t k = chain(key, toks + l);
            auto it = by_key_.find(k);
            if (it == by_key_.end()) break;
            const int p = it->second;
            const Page &g = pg_[(size_t)p];
            if (!g.cached || g.parent != parent || g.parent_gen != pgen || !same(g.toks, toks + l, kPageRows)) break;
            ref(p);
            m.full.push_back(p);
            parent = p;
            pgen = g.gen;
            key = k;
            l += kPageRows;
        }
        auto ch = children_.find(child_key(parent, pgen));
        if (ch != children_.end()) {
            for (int c : ch->second) {
                const Page &g = pg_[(size_t)c];
                int r = 0;
                while (r < kPageRows && l + r < limit && g.toks[r] == toks[l + r]) r++;
                if (r > m.src_rows) {
                    m.src_rows = r;
                    m.src = c;
                }
            }
        }
        m.rows = l + m.src_rows;
        return m;
    }

  private:
    static constexpr uint64_t kRootKey = 0x9E3779B97F4A7C15ull;
    struct Page {
        int ref = 0;
        uint32_t gen = 0;  // bumped on every reuse: a child's parent link names (page, gen)
        bool cached = false, in_lru = false;
        uint64_t key = 0;
        int parent = -1;
        uint32_t parent_gen = 0;
        int toks[kPageRows] = {};
        std::list<int>::iterator lru;
    };

    static uint64_t mix(uint64_t h, uint64_t v) {
        h ^= v + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
        h *= 0xBF58476D1CE4E5B9ull;
        return h ^ (h >> 31);
    }
    static uint64_t chain(uint64_t h, const int *toks) {
        for (int i = 0; i < kPageRows; i++) h = mix(h, (uint32_t)toks[i]);
        return h;
    }
    static long long child_key(int parent, uint32_t gen) { return ((long long)(parent + 1) << 32) | gen; }
    static bool same(const int *a, const int *b, int n) {
        for (int i = 0; i < n; i++)
            if (a[i] != b[i]) return false;
        return true;
    }
    // The least recently used idle cached page leaves the cache for reuse.
    void evict(int p) {
        unregister(p, false);
        evictions_++;
    }
    // Drop p from the cache; an idle page goes to the free list unless the
    // caller reuses it at once.
    void unregister(int p, bool to_free = true) {
        Page &g = pg_[(size_t)p];
        if (g.in_lru) {
            lru_.erase(g.lru);
            g.in_lru = false;
        }
        by_key_.erase(g.key);
        auto ch = children_.find(child_key(g.parent, g.parent_gen));
        if (ch != children_.end()) {
            auto &v = ch->second;
            for (size_t i = 0; i < v.size(); i++)
                if (v[i] == p) {
                    v[i] = v.back();
                    v.pop_back();
                    break;
                }
            if (v.empty()) children_.erase(ch);
        }
        children_.erase(child_key(p, g.gen));  // its children can no longer be reached through it
        g.cached = false;
        g.gen++;
        if (to_free && g.ref == 0) free_.push_back(p);
    }

    std::vector<Page> pg_;
    std::vector<int> free_;
    std::list<int> lru_;
    std::unordered_map<uint64_t, int> by_key_;
    std::unordered_map<long long, std::vector<int>> children_;
    long long evictions_ = 0;
};

}  // namespace hyk
