// prefix_cache.cpp — page-refcounted prompt-prefix cache (host side, single-threaded).
//
// The reference keeps a trie of cached prompt prefixes whose entries each own a private copy of
// the model state (src/server/prefix_state_cache.zig:21-213 index, :292-567 cache). A hit copies
// the entry's linear state into the request's work state and reads the entry's KV as a second
// source; storing copies the work state's new KV rows into the entry
// (state.zig:124-230 via prefix_state_cache.zig:344-424).
//
// Here KV lives in one paged pool shared by every sequence and every entry, so an entry is a
// list of page ids and a hit is a refcount increment: pgc_prefix_cache_fork hands the request the
// entry's pages, and pgc_page_pool_make_writable copies a page only when a sequence is about to
// write into a page that someone else still holds (in practice the one partial page at the end of
// the matched prefix). Storing a prefix adopts the work sequence's pages (no copy). The same page
// ids index the hidden-row pool, so MTP hidden rows are shared the same way. Linear (recurrent and
// conv) state is not pageable; each entry owns a state slot and the caller copies that state
// (pgc_copy_regions) where the reference copies it.
//
// The cache policy is the reference's, kept exactly so that its tests transcribe: token-level
// longest-prefix match, the reserved-token budget (capacity = max(len, prefill chunk)), LRU
// eviction of unpinned entries that never evicts the entry being extended, dense entry indexes
// that shift down when an earlier entry is removed, and the hidden-row validity rules.
#include <algorithm>
#include <cstring>
#include <new>
#include <unordered_map>
#include <vector>

#include "../../include/peregrine_cuda.h"

struct pgc_page_pool {
    std::vector<int32_t> ref;        // refcount per page (0 = free)
    std::vector<int32_t> free_list;  // stack of free page ids, lowest id on top
    int attached = 0;                // caches built on this pool
    bool destroy_requested = false;  // destroyed while caches were attached: freed with the last
};

namespace {

int pool_alloc(pgc_page_pool *p, int32_t n, int32_t *out) {
    if ((int64_t)p->free_list.size() < n) return PGC_ERR_CAPACITY;
    for (int32_t i = 0; i < n; ++i) {
        const int32_t page = p->free_list.back();
        p->free_list.pop_back();
        p->ref[page] = 1;
        out[i] = page;
    }
    return PGC_OK;
}

bool pages_live(const pgc_page_pool *p, const int32_t *pages, int64_t n) {
    for (int64_t i = 0; i < n; ++i)
        if (pages[i] < 0 || pages[i] >= (int32_t)p->ref.size() || p->ref[pages[i]] <= 0) return false;
    return true;
}

void pool_retain(pgc_page_pool *p, const int32_t *pages, int64_t n) {
    for (int64_t i = 0; i < n; ++i) ++p->ref[pages[i]];
}

void pool_release(pgc_page_pool *p, const int32_t *pages, int64_t n) {
    for (int64_t i = 0; i < n; ++i)
        if (--p->ref[pages[i]] == 0) p->free_list.push_back(pages[i]);
}

// ---------------------------------------------------------------------------- prefix index
// Same contract as the reference index (prefix_state_cache.zig:21-213) — insert a token
// sequence with an entry index, exact and longest-prefix lookup, removal that prunes nodes
// carrying nothing — but path-compressed: a node holds the run of tokens on the edge from its
// parent, so a lookup compares token spans instead of one hash probe per token (a 24k-token
// prompt walks a handful of nodes). Nodes keep their id while the tree is re-shaped (a split
// inserts the new node above; a merge folds the parent into its only child), so an entry can
// remember the id of the node it ends at. Children are found through one hash map keyed by
// (node, first token of the child's run).
class Trie {
  public:
    void clear() {
        nodes_.clear();
        free_.clear();
        child_.clear();
    }

    // Node ending exactly at `tokens` (splitting an edge or adding a leaf as needed), whose
    // entry is set to `entry`.
    int32_t insert(const uint32_t *tokens, uint64_t n, int64_t entry) {
        ensure_root();
        int32_t node = 0;
        uint64_t i = 0;
        while (i < n) {
            auto it = child_.find(edge(node, tokens[i]));
            if (it == child_.end()) {
                const int32_t leaf = alloc(node, tokens + i, n - i);
                child_.emplace(edge(node, tokens[i]), leaf);
                ++nodes_[node].children;
                node = leaf;
                i = n;
                break;
            }
            const int32_t c = it->second;
            const uint64_t l = common(nodes_[c].run, tokens + i, n - i);
            if (l < nodes_[c].run.size()) {
                split(c, l);
                node = nodes_[c].parent;  // the new node ending after l tokens
            } else {
                node = c;
            }
            i += l;
        }
        nodes_[node].entry = entry;
        return node;
    }

    int32_t find_node(const uint32_t *tokens, uint64_t n) const {
        if (nodes_.empty()) return -1;
        int32_t node = 0;
        uint64_t i = 0;
        while (i < n) {
            auto it = child_.find(edge(node, tokens[i]));
            if (it == child_.end()) return -1;
            const Node &c = nodes_[it->second];
            if (c.run.size() > n - i || common(c.run, tokens + i, n - i) != c.run.size()) return -1;
            node = it->second;
            i += c.run.size();
        }
        return node;
    }

    void remove(const uint32_t *tokens, uint64_t n) {
        const int32_t node = find_node(tokens, n);
        if (node < 0) return;
        nodes_[node].entry = -1;
        prune(node);
    }

    // Longest prompt prefix ending at a node that carries an entry (findLongest).
    bool find_longest(const uint32_t *prompt, uint64_t n, int64_t *entry, uint64_t *len) const {
        if (nodes_.empty()) return false;
        int32_t node = 0;
        uint64_t i = 0;
        bool found = false;
        while (i < n) {
            auto it = child_.find(edge(node, prompt[i]));
            if (it == child_.end()) break;
            const Node &c = nodes_[it->second];
            if (c.run.size() > n - i || common(c.run, prompt + i, n - i) != c.run.size()) break;
            node = it->second;
            i += c.run.size();
            if (c.entry >= 0) {
                *entry = c.entry;
                *len = i;
                found = true;
            }
        }
        return found;
    }

    int64_t entry_at(int32_t node) const { return node < 0 ? -1 : nodes_[node].entry; }
    void set_entry(int32_t node, int64_t entry) { nodes_[node].entry = entry; }
    uint64_t live_nodes() const { return nodes_.size() - free_.size(); }

  private:
    struct Node {
        int32_t parent = -1;
        int32_t children = 0;
        int64_t entry = -1;
        std::vector<uint32_t> run;  // tokens on the edge from the parent
    };

    static uint64_t edge(int32_t parent, uint32_t token) {
        return ((uint64_t)(uint32_t)parent << 32) | token;
    }

    static uint64_t common(const std::vector<uint32_t> &run, const uint32_t *t, uint64_t n) {
        const uint64_t m = std::min<uint64_t>(run.size(), n);
        // whole runs usually match: compare 1024-token blocks with memcmp, then finish the
        // first differing block token by token
        uint64_t i = 0;
        while (i + 1024 <= m && std::memcmp(run.data() + i, t + i, 1024 * 4) == 0) i += 1024;
        while (i < m && run[i] == t[i]) ++i;
        return i;
    }

    void ensure_root() {
        if (nodes_.empty()) nodes_.push_back(Node{});
    }

    int32_t alloc(int32_t parent, const uint32_t *run, uint64_t len) {
        Node nd;
        nd.parent = parent;
        nd.run.assign(run, run + len);
        if (!free_.empty()) {
            const int32_t i = free_.back();
            free_.pop_back();
            nodes_[i] = std::move(nd);
            return i;
        }
        nodes_.push_back(std::move(nd));
        return (int32_t)nodes_.size() - 1;
    }

    // New node above c holding the first l tokens of c's run; c keeps its id.
    void split(int32_t c, uint64_t l) {
        const int32_t parent = nodes_[c].parent;
        const uint32_t first = nodes_[c].run[0];
        const int32_t mid = alloc(parent, nodes_[c].run.data(), l);  // may move nodes_
        Node &cn = nodes_[c];
        cn.run.erase(cn.run.begin(), cn.run.begin() + (int64_t)l);
        cn.parent = mid;
        nodes_[mid].children = 1;
        child_[edge(parent, first)] = mid;
        child_.emplace(edge(mid, cn.run[0]), c);
    }

    void unlink(int32_t node) {
        Node &nd = nodes_[node];
        child_.erase(edge(nd.parent, nd.run[0]));
        --nodes_[nd.parent].children;
        nodes_[node] = Node{};
        free_.push_back(node);
    }

    // After node lost its entry: drop it if it is a leaf, fold it into its only child if it
    // has one, then do the same for a parent left without entry and with at most one child.
    void prune(int32_t node) {
        while (node != 0) {
            Node &nd = nodes_[node];
            if (nd.entry >= 0 || nd.children > 1) return;
            const int32_t parent = nd.parent;
            if (nd.children == 0) {
                unlink(node);
                node = parent;
                continue;
            }
            // one child: the child absorbs this node's run and takes its place under parent
            int32_t only = -1;
            for (const auto &kv : child_)
                if ((int32_t)(kv.first >> 32) == node) {
                    only = kv.second;
                    break;
                }
            fold_into_child(node, only);
            return;
        }
    }

    void fold_into_child(int32_t node, int32_t only) {
        Node &nd = nodes_[node];
        Node &ch = nodes_[only];
        const int32_t parent = nd.parent;
        child_.erase(edge(node, ch.run[0]));
        child_[edge(parent, nd.run[0])] = only;
        ch.run.insert(ch.run.begin(), nd.run.begin(), nd.run.end());
        ch.parent = parent;
        nodes_[node] = Node{};
        free_.push_back(node);
    }

    std::vector<Node> nodes_;
    std::vector<int32_t> free_;
    std::unordered_map<uint64_t, int32_t> child_;
};

struct Entry {
    std::vector<uint32_t> tokens;
    std::vector<int32_t> pages;  // ceil(len / page_tokens) page ids, one reference each
    uint64_t capacity = 0;       // reserved tokens (the reference's cached_state.max_seq)
    int32_t state_slot = -1;
    int32_t node = -1;           // trie node carrying this entry, -1 while not indexed
    bool pinned = false;
    bool hidden_valid = false;
    bool next_valid = false;
    uint32_t next_token = 0;
    uint64_t last_access = 0;
    uint64_t hits = 0;
};

}  // namespace

struct pgc_prefix_cache {
    pgc_page_pool *pool = nullptr;
    int32_t page_tokens = 16;
    uint64_t max_tokens = 0;
    uint64_t initial_state_tokens = 0;
    std::vector<Entry> entries;
    Trie index;
    std::vector<int32_t> free_slots;  // linear-state slots not owned by an entry
    uint64_t resident = 0, reserved = 0;
    int64_t active = -1;
    uint64_t clock = 0;
    uint64_t hits = 0, misses = 0, hit_tokens = 0, computed_tokens = 0, evictions = 0;
    bool track_hidden = false;

    int64_t pages_for(uint64_t tokens) const { return (int64_t)((tokens + page_tokens - 1) / page_tokens); }
    uint64_t next_access() { return ++clock; }

    void set_pages(Entry &e, const int32_t *pages, int64_t n) {
        // retain first: the new list usually shares its leading pages with the old one
        pool_retain(pool, pages, n);
        if (!e.pages.empty()) pool_release(pool, e.pages.data(), (int64_t)e.pages.size());
        e.pages.assign(pages, pages + n);
    }

    // prefix_state_cache.zig:295-313 (removeEntry): later indexes shift down by one.
    void remove_entry(int64_t i) {
        Entry &e = entries[i];
        if (e.node >= 0 && index.entry_at(e.node) == i) index.remove(e.tokens.data(), e.tokens.size());
        resident = resident >= e.tokens.size() ? resident - e.tokens.size() : 0;
        reserved = reserved >= e.capacity ? reserved - e.capacity : 0;
        if (!e.pages.empty()) pool_release(pool, e.pages.data(), (int64_t)e.pages.size());
        if (e.state_slot >= 0) free_slots.push_back(e.state_slot);
        entries.erase(entries.begin() + i);
        for (int64_t j = i; j < (int64_t)entries.size(); ++j)
            if (entries[j].node >= 0 && index.entry_at(entries[j].node) == j + 1)
                index.set_entry(entries[j].node, j);
        if (active == i) active = -1;
        else if (active > i) --active;
    }

    // prefix_state_cache.zig:551-561: least recently used unpinned entry other than `preserve`.
    int64_t evictable(int64_t preserve) const {
        int64_t victim = -1;
        for (int64_t i = 0; i < (int64_t)entries.size(); ++i) {
            if (i == preserve || entries[i].pinned) continue;
            if (victim < 0 || entries[i].last_access < entries[victim].last_access) victim = i;
        }
        return victim;
    }

    void evict(int64_t victim, int64_t *preserve) {
        remove_entry(victim);
        if (*preserve >= 0 && victim < *preserve) --*preserve;
        ++evictions;
    }

    // prefix_state_cache.zig:530-545 (ensureReservedTokenBudget).
    int ensure_budget(int64_t *preserve, uint64_t additional) {
        if (additional > max_tokens) return PGC_ERR_BOUNDS;
        while (reserved + additional > max_tokens) {
            const int64_t v = evictable(*preserve);
            if (v < 0) return PGC_ERR_BOUNDS;
            evict(v, preserve);
        }
        return PGC_OK;
    }

    // Frees entries (LRU, unpinned) until `need` pages are free in the pool.
    int ensure_pages(int64_t *preserve, int64_t need) {
        while ((int64_t)pool->free_list.size() < need) {
            const int64_t v = evictable(*preserve);
            if (v < 0) return PGC_ERR_CAPACITY;
            evict(v, preserve);
        }
        return PGC_OK;
    }

    int ensure_slot(int64_t *preserve) {
        while (free_slots.empty()) {
            const int64_t v = evictable(*preserve);
            if (v < 0) return PGC_ERR_CAPACITY;
            evict(v, preserve);
        }
        return PGC_OK;
    }

    // prefix_state_cache.zig:503-524 (replaceEntryPrefix).
    int replace_prefix(int64_t *preserved, const uint32_t *ids, uint64_t n, bool pin) {
        const uint64_t old_cap = entries[*preserved].capacity;
        if (n > old_cap) {
            const int st = ensure_budget(preserved, n - old_cap);
            if (st != PGC_OK) return st;
        }
        Entry &e = entries[*preserved];
        const uint64_t old_len = e.tokens.size();
        const uint64_t new_cap = std::max(old_cap, n);
        reserved = reserved - old_cap + new_cap;
        e.capacity = new_cap;
        e.tokens.assign(ids, ids + n);
        e.pinned = e.pinned || pin;
        resident = resident - old_len + n;
        return PGC_OK;
    }

    // prefix_state_cache.zig:455-501 (prepareEntry).
    int prepare(const uint32_t *ids, uint64_t n, int64_t reuse_index, bool pin, int64_t *out) {
        if (n == 0 || n > max_tokens) return PGC_ERR_BOUNDS;
        const int64_t exact = index.entry_at(index.find_node(ids, n));
        if (exact >= 0) {
            int64_t keep = exact;
            const int st = replace_prefix(&keep, ids, n, pin);
            if (st != PGC_OK) return st;
            *out = keep;
            return PGC_OK;
        }
        if (reuse_index >= 0) {
            int64_t keep = reuse_index;
            const std::vector<uint32_t> old_tokens = entries[keep].tokens;
            const int32_t old_node = entries[keep].node;
            entries[keep].node = index.insert(ids, n, keep);
            const int st = replace_prefix(&keep, ids, n, pin);
            if (st != PGC_OK) {
                index.remove(ids, n);
                entries[keep].node = old_node;
                return st;
            }
            index.remove(old_tokens.data(), old_tokens.size());
            *out = keep;
            return PGC_OK;
        }
        int64_t none = -1;
        const uint64_t cap = std::max(n, initial_state_tokens);
        int st = ensure_budget(&none, cap);
        if (st == PGC_OK) st = ensure_slot(&none);
        if (st != PGC_OK) return st;
        Entry e;
        e.tokens.assign(ids, ids + n);
        e.capacity = cap;
        e.pinned = pin;
        e.last_access = next_access();
        e.state_slot = free_slots.back();
        free_slots.pop_back();
        const int64_t idx = (int64_t)entries.size();
        e.node = index.insert(ids, n, idx);
        entries.push_back(std::move(e));
        resident += n;
        reserved += cap;
        *out = idx;
        return PGC_OK;
    }

    void touch(int64_t i) {
        if (i < 0 || i >= (int64_t)entries.size()) return;
        Entry &e = entries[i];
        e.last_access = next_access();
        ++e.hits;
        active = i;
    }

    void clear_all() {
        for (Entry &e : entries) {
            if (!e.pages.empty()) pool_release(pool, e.pages.data(), (int64_t)e.pages.size());
            if (e.state_slot >= 0) free_slots.push_back(e.state_slot);
        }
        entries.clear();
        index.clear();
        resident = reserved = 0;
        active = -1;
    }

    bool valid(const pgc_match *m) const {
        return m && m->index >= 0 && m->index < (int64_t)entries.size();
    }
};

extern "C" {

// ------------------------------------------------------------------------------ page pool

pgc_page_pool *pgc_page_pool_create(int32_t num_pages) {
    if (num_pages <= 0) return nullptr;
    pgc_page_pool *p = new (std::nothrow) pgc_page_pool;
    if (!p) return nullptr;
    p->ref.assign(num_pages, 0);
    p->free_list.resize(num_pages);
    for (int32_t i = 0; i < num_pages; ++i) p->free_list[i] = num_pages - 1 - i;
    return p;
}

void pgc_page_pool_destroy(pgc_page_pool *pool) {
    if (!pool) return;
    if (pool->attached > 0) pool->destroy_requested = true;  // the last cache frees it
    else delete pool;
}

int pgc_page_pool_alloc(pgc_page_pool *pool, int32_t n, int32_t *pages_out) {
    if (!pool || n < 0 || (n > 0 && !pages_out)) return PGC_ERR_INVALID;
    return pool_alloc(pool, n, pages_out);
}

int pgc_page_pool_retain(pgc_page_pool *pool, const int32_t *pages, int32_t n) {
    if (!pool || n < 0 || (n > 0 && !pages)) return PGC_ERR_INVALID;
    if (!pages_live(pool, pages, n)) return PGC_ERR_BOUNDS;
    pool_retain(pool, pages, n);
    return PGC_OK;
}

int pgc_page_pool_release(pgc_page_pool *pool, const int32_t *pages, int32_t n) {
    if (!pool || n < 0 || (n > 0 && !pages)) return PGC_ERR_INVALID;
    if (!pages_live(pool, pages, n)) return PGC_ERR_BOUNDS;
    // a page listed twice must hold two references: drop them all, and undo everything if
    // one went below zero
    for (int32_t i = 0; i < n; ++i) {
        if (--pool->ref[pages[i]] < 0) {
            for (int32_t j = 0; j <= i; ++j) ++pool->ref[pages[j]];
            return PGC_ERR_BOUNDS;
        }
    }
    for (int32_t i = 0; i < n; ++i)
        if (pool->ref[pages[i]] == 0) {
            pool->free_list.push_back(pages[i]);
            pool->ref[pages[i]] = -1;  // listed again below: push once
        }
    for (int32_t i = 0; i < n; ++i)
        if (pool->ref[pages[i]] < 0) pool->ref[pages[i]] = 0;
    return PGC_OK;
}

int32_t pgc_page_pool_refcount(const pgc_page_pool *pool, int32_t page) {
    if (!pool || page < 0 || page >= (int32_t)pool->ref.size()) return PGC_ERR_BOUNDS;
    return pool->ref[page];
}

int32_t pgc_page_pool_free_pages(const pgc_page_pool *pool) {
    return pool ? (int32_t)pool->free_list.size() : PGC_ERR_INVALID;
}

int pgc_page_pool_make_writable(pgc_page_pool *pool, int32_t *table, int32_t slot,
                                int32_t *src_page, int32_t *dst_page) {
    if (!pool || !table || slot < 0 || !src_page || !dst_page) return PGC_ERR_INVALID;
    const int32_t page = table[slot];
    if (!pages_live(pool, &page, 1)) return PGC_ERR_BOUNDS;
    if (pool->ref[page] == 1) {
        *src_page = *dst_page = page;
        return PGC_OK;
    }
    int32_t fresh;
    const int st = pool_alloc(pool, 1, &fresh);
    if (st != PGC_OK) return st;
    --pool->ref[page];
    table[slot] = fresh;
    *src_page = page;
    *dst_page = fresh;
    return PGC_OK;
}

// ---------------------------------------------------------------------------- prefix cache

pgc_prefix_cache *pgc_prefix_cache_create(pgc_page_pool *pool, int32_t page_tokens,
                                          uint64_t max_tokens, uint64_t prefill_chunk_tokens,
                                          int32_t state_slots) {
    if (!pool || page_tokens <= 0 || max_tokens == 0 || state_slots <= 0) return nullptr;
    pgc_prefix_cache *c = new (std::nothrow) pgc_prefix_cache;
    if (!c) return nullptr;
    c->pool = pool;
    ++pool->attached;
    c->page_tokens = page_tokens;
    c->max_tokens = max_tokens;
    c->initial_state_tokens = std::min(max_tokens, prefill_chunk_tokens);
    c->free_slots.resize(state_slots);
    for (int32_t i = 0; i < state_slots; ++i) c->free_slots[i] = state_slots - 1 - i;
    return c;
}

void pgc_prefix_cache_destroy(pgc_prefix_cache *cache) {
    if (!cache) return;
    cache->clear_all();
    pgc_page_pool *pool = cache->pool;
    delete cache;
    if (--pool->attached == 0 && pool->destroy_requested) delete pool;
}

void pgc_prefix_cache_clear_all(pgc_prefix_cache *cache) {
    if (cache) cache->clear_all();
}

void pgc_prefix_cache_enable_hidden_tracking(pgc_prefix_cache *cache) {
    if (cache) cache->track_hidden = true;
}

int pgc_prefix_cache_find(const pgc_prefix_cache *cache, const uint32_t *prompt, uint64_t n,
                          pgc_match *out) {
    if (!cache || !out || (n > 0 && !prompt)) return PGC_ERR_INVALID;
    out->index = -1;
    out->len = 0;
    int64_t e;
    uint64_t len;
    if (!cache->index.find_longest(prompt, n, &e, &len)) return 0;
    out->index = e;
    out->len = (int64_t)len;
    return 1;
}

int pgc_prefix_cache_contains(const pgc_prefix_cache *cache, const uint32_t *prompt, uint64_t n,
                              uint64_t prefix_len) {
    if (!cache || (n > 0 && !prompt)) return PGC_ERR_INVALID;
    if (prefix_len == 0) return 1;
    if (prefix_len > n) return 0;
    return cache->index.entry_at(cache->index.find_node(prompt, prefix_len)) >= 0 ? 1 : 0;
}

void pgc_prefix_cache_touch(pgc_prefix_cache *cache, pgc_match match) {
    if (cache) cache->touch(match.index);
}

void pgc_prefix_cache_record_hit(pgc_prefix_cache *cache, uint64_t reused_tokens) {
    if (!cache) return;
    ++cache->hits;
    cache->hit_tokens += reused_tokens;
}

void pgc_prefix_cache_record_miss(pgc_prefix_cache *cache) {
    if (cache) ++cache->misses;
}

void pgc_prefix_cache_record_computed(pgc_prefix_cache *cache, uint64_t tokens) {
    if (cache) cache->computed_tokens += tokens;
}

int pgc_prefix_cache_stats(const pgc_prefix_cache *cache, pgc_prefix_stats *out) {
    if (!cache || !out) return PGC_ERR_INVALID;
    out->hits = cache->hits;
    out->misses = cache->misses;
    out->hit_tokens = cache->hit_tokens;
    out->computed_tokens = cache->computed_tokens;
    out->reserved_tokens = cache->reserved;
    out->resident_tokens = cache->resident;
    out->max_tokens = cache->max_tokens;
    out->entry_count = cache->entries.size();
    out->pinned_count = 0;
    for (const Entry &e : cache->entries) out->pinned_count += e.pinned ? 1 : 0;
    out->evictions = cache->evictions;
    out->active_index = cache->active;
    out->trie_nodes = cache->index.live_nodes();
    return PGC_OK;
}

int pgc_prefix_cache_entry(const pgc_prefix_cache *cache, int64_t index, pgc_prefix_entry *out,
                           uint32_t *tokens_out, uint64_t tokens_cap, int32_t *pages_out,
                           int64_t pages_cap) {
    if (!cache || !out) return PGC_ERR_INVALID;
    if (index < 0 || index >= (int64_t)cache->entries.size()) return PGC_ERR_BOUNDS;
    const Entry &e = cache->entries[index];
    out->token_count = e.tokens.size();
    out->page_count = (int64_t)e.pages.size();
    out->capacity = e.capacity;
    out->state_slot = e.state_slot;
    out->pinned = e.pinned;
    out->hidden_valid = e.hidden_valid;
    out->next_token_valid = e.next_valid;
    out->next_token = e.next_token;
    out->last_access = e.last_access;
    out->hits = e.hits;
    if (tokens_out) {
        if (tokens_cap < e.tokens.size()) return PGC_ERR_BOUNDS;
        std::memcpy(tokens_out, e.tokens.data(), e.tokens.size() * 4);
    }
    if (pages_out) {
        if (pages_cap < (int64_t)e.pages.size()) return PGC_ERR_BOUNDS;
        std::memcpy(pages_out, e.pages.data(), e.pages.size() * 4);
    }
    return PGC_OK;
}

int pgc_prefix_cache_remove(pgc_prefix_cache *cache, int64_t index) {
    if (!cache) return PGC_ERR_INVALID;
    if (index < 0 || index >= (int64_t)cache->entries.size()) return PGC_OK;  // as the reference
    cache->remove_entry(index);
    return PGC_OK;
}

int pgc_prefix_cache_start_direct(pgc_prefix_cache *cache, const uint32_t *ids, uint64_t n,
                                  int pinned, pgc_match *out) {
    if (!cache || !out || (n > 0 && !ids)) return PGC_ERR_INVALID;
    if (n == 0 || n > cache->max_tokens) return PGC_ERR_BOUNDS;
    const int64_t need = cache->pages_for(n);
    // fresh pages: the caller prefills straight into them, and an older entry's pages may still
    // be read by sequences that forked from it
    int64_t none = -1;
    int st = cache->ensure_pages(&none, need);
    if (st != PGC_OK) return st;
    std::vector<int32_t> pages(need);
    st = pool_alloc(cache->pool, (int32_t)need, pages.data());
    if (st != PGC_OK) return st;
    int64_t idx;
    st = cache->prepare(ids, n, -1, pinned != 0, &idx);
    if (st != PGC_OK) {
        pool_release(cache->pool, pages.data(), need);
        return st;
    }
    Entry &e = cache->entries[idx];
    if (!e.pages.empty()) pool_release(cache->pool, e.pages.data(), (int64_t)e.pages.size());
    e.pages = std::move(pages);
    e.next_valid = false;
    out->index = idx;
    out->len = (int64_t)n;
    return PGC_OK;
}

int pgc_prefix_cache_finish_direct(pgc_prefix_cache *cache, pgc_match match, uint32_t next_token) {
    if (!cache) return PGC_ERR_INVALID;
    if (!cache->valid(&match)) return PGC_ERR_BOUNDS;
    Entry &e = cache->entries[match.index];
    e.next_token = next_token;
    e.next_valid = true;
    cache->touch(match.index);
    return PGC_OK;
}

int pgc_prefix_cache_set_hidden_valid(pgc_prefix_cache *cache, pgc_match match, int valid) {
    if (!cache) return PGC_ERR_INVALID;
    if (!cache->valid(&match)) return PGC_ERR_BOUNDS;
    if (cache->track_hidden) cache->entries[match.index].hidden_valid = valid != 0;
    return PGC_OK;
}

int pgc_prefix_cache_store(pgc_prefix_cache *cache, const uint32_t *ids, uint64_t n,
                           const pgc_match *reuse, const int32_t *work_table, int64_t work_pages,
                           int suffix_hidden, const uint32_t *next_token, int pinned,
                           pgc_match *out, int *copy_linear_state) {
    if (!cache || !out || (n > 0 && !ids) || !work_table) return PGC_ERR_INVALID;
    if (n == 0 || n > cache->max_tokens) return PGC_ERR_BOUNDS;
    const int64_t need = cache->pages_for(n);
    if (work_pages < need) return PGC_ERR_BOUNDS;
    if (!pages_live(cache->pool, work_table, need)) return PGC_ERR_BOUNDS;
    if (reuse && (reuse->index < 0 || reuse->index >= (int64_t)cache->entries.size()))
        return PGC_ERR_BOUNDS;
    const int64_t reuse_index = reuse ? reuse->index : -1;
    const bool had_exact = cache->index.entry_at(cache->index.find_node(ids, n)) >= 0;
    int64_t idx;
    const int st = cache->prepare(ids, n, reuse_index, pinned != 0, &idx);
    if (st != PGC_OK) return st;
    Entry &e = cache->entries[idx];
    const uint64_t reuse_len =
        reuse ? std::min<uint64_t>((uint64_t)std::max<int64_t>(reuse->len, 0), n) : 0;
    // The work sequence's pages already hold rows [0, n): the prefix rows it forked from this
    // (or another) entry and the rows it computed. Adopting them replaces the reference's copy of
    // the suffix range and, for a fresh entry, of the whole prefix.
    cache->set_pages(e, work_table, need);
    if (copy_linear_state)
        *copy_linear_state = !had_exact && ((reuse && n > reuse_len) || reuse_len == 0);
    if (cache->track_hidden) {
        // prefix_state_cache.zig:378-412: valid when the reused rows were valid and the suffix
        // rows are real (or absent). `e` is the reused entry after any index shift.
        const bool reuse_valid = reuse_len != 0 ? e.hidden_valid : false;
        const uint64_t suffix_rows = n - reuse_len;
        const bool prefix_half = reuse_len == 0 || reuse_valid;
        const bool suffix_half = suffix_rows == 0 || suffix_hidden != 0;
        e.hidden_valid = prefix_half && suffix_half;
    }
    if (next_token) {
        e.next_token = *next_token;
        e.next_valid = true;
    } else {
        e.next_valid = false;
    }
    cache->touch(idx);
    out->index = idx;
    out->len = (int64_t)n;
    return PGC_OK;
}

int pgc_prefix_cache_fork(pgc_prefix_cache *cache, pgc_match match, int32_t *table_out,
                          int64_t table_cap, int64_t *pages_out) {
    if (!cache || !table_out || !pages_out) return PGC_ERR_INVALID;
    if (!cache->valid(&match)) return PGC_ERR_BOUNDS;
    const Entry &e = cache->entries[match.index];
    if (match.len <= 0 || (uint64_t)match.len > e.tokens.size()) return PGC_ERR_BOUNDS;
    const int64_t n = cache->pages_for((uint64_t)match.len);
    if (table_cap < n) return PGC_ERR_BOUNDS;
    pool_retain(cache->pool, e.pages.data(), n);
    std::memcpy(table_out, e.pages.data(), n * 4);
    *pages_out = n;
    return PGC_OK;
}

int pgc_prefix_cache_evict_for_pages(pgc_prefix_cache *cache, int32_t need_free) {
    if (!cache || need_free < 0) return PGC_ERR_INVALID;
    int64_t none = -1;
    return cache->ensure_pages(&none, need_free);
}

int pgc_prefix_cache_load_slot(pgc_prefix_cache *cache, const uint32_t *ids, uint64_t n,
                               pgc_match *out) {
    if (!cache || !out || (n > 0 && !ids)) return PGC_ERR_INVALID;
    cache->clear_all();
    if (n == 0 || n > cache->max_tokens) return PGC_ERR_BOUNDS;
    const int64_t need = cache->pages_for(n);
    Entry e;
    e.pages.resize(need);
    const int st = pool_alloc(cache->pool, (int32_t)need, e.pages.data());
    if (st != PGC_OK) return st;
    e.tokens.assign(ids, ids + n);
    e.capacity = std::max(n, cache->initial_state_tokens);
    e.pinned = true;
    e.last_access = cache->next_access();
    e.state_slot = cache->free_slots.back();
    cache->free_slots.pop_back();
    cache->entries.push_back(std::move(e));
    cache->resident = n;
    cache->reserved = cache->entries.back().capacity;
    cache->active = (int64_t)cache->entries.size() - 1;
    out->index = cache->active;
    out->len = (int64_t)n;
    return PGC_OK;
}

int pgc_prefix_cache_finish_loaded(pgc_prefix_cache *cache, pgc_match match) {
    if (!cache) return PGC_ERR_INVALID;
    if (!cache->valid(&match)) return PGC_ERR_INVALID;
    Entry &e = cache->entries[match.index];
    if ((int64_t)e.tokens.size() != match.len) return PGC_ERR_BOUNDS;
    e.node = cache->index.insert(e.tokens.data(), e.tokens.size(), match.index);
    return PGC_OK;
}

int pgc_prefix_cache_persisted(const pgc_prefix_cache *cache, pgc_match *out) {
    if (!cache || !out) return PGC_ERR_INVALID;
    int64_t best = -1;
    if (cache->active >= 0 && cache->active < (int64_t)cache->entries.size()) {
        best = cache->active;
    } else {
        for (int64_t i = 0; i < (int64_t)cache->entries.size(); ++i) {
            if (cache->entries[i].tokens.empty()) continue;
            if (best < 0 || cache->entries[i].last_access > cache->entries[best].last_access) best = i;
        }
    }
    out->index = best;
    out->len = best >= 0 ? (int64_t)cache->entries[best].tokens.size() : 0;
    return best >= 0 ? 1 : 0;
}

}  // extern "C"
