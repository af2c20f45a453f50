"""Page-refcounted prefix cache (csrc/prefix_cache.cpp).

CPU: the reference's own cache tests transcribed one for one
(src/server/prefix_state_cache.zig:588-1201; entries are made with startDirectEntry +
finishDirectEntry as its addTestEntry does, a work state is a block table of pool pages), the
page pool's refcount / copy-on-write contract, and a seeded random walk that checks the
bookkeeping invariants after every operation.
GPU: two requests fork one cached prefix whose last page is partial, each copies that page on
write and fills its own suffix; both sequences and the cached entry then read back bit-exact and
decode within the attention tolerance of the oracle."""
import numpy as np
import pytest

from _util import D, NKV, PAGE


@pytest.fixture(scope="module")
def pc():
    from peregrine_b200 import build
    build.build()
    from peregrine_b200 import prefix_cache
    return prefix_cache


def _cache(pc, max_tokens, chunk, pages=256, slots=64):
    pool = pc.PagePool(pages)
    return pool, pc.PrefixCache(pool, max_tokens, chunk, state_slots=slots)


def _add(cache, tokens, pinned, next_token):
    # addTestEntry (prefix_state_cache.zig:576-586)
    m = cache.start_direct_entry(tokens, pinned)
    cache.finish_direct_entry(m, next_token)
    return m


def _work_table(pool, cache, reuse, n):
    """A work sequence's block table for n tokens: the reused entry's pages (forked) plus fresh
    ones, with the partial boundary page made writable."""
    table = np.zeros(0, np.int32)
    if reuse is not None:
        table = cache.fork(reuse)
        if reuse.len % PAGE:
            pool.make_writable(table, len(table) - 1)
    need = -(-n // PAGE) - len(table)
    return np.concatenate([table, pool.alloc(need)]) if need > 0 else table


# ------------------------------------------------------------------ reference tests, transcribed

def test_keeps_multiple_exact_prefix_entries(pc):
    _, c = _cache(pc, 12, 4)
    _add(c, [1, 2, 3], False, 10)
    _add(c, [1, 2, 3, 4], False, 11)
    _add(c, [9, 8], False, 12)
    s = c.stats()
    assert (s.entry_count, s.resident_tokens, s.reserved_tokens) == (3, 9, 12)
    longest = c.find_prefix([1, 2, 3, 4, 5])
    assert longest.len == 4 and c.cached_next_token(longest) == 11
    assert c.find_prefix([1, 2, 9]) is None
    assert c.contains_prompt_prefix([1, 2, 3, 4, 5], 3)


def test_evicts_least_recently_used_unpinned_entries(pc):
    _, c = _cache(pc, 8, 4)
    first = _add(c, [1, 2, 3], False, 10)
    _add(c, [4, 5, 6], False, 11)
    c.touch(first)
    _add(c, [7, 8, 9], False, 12)
    s = c.stats()
    assert (s.entry_count, s.resident_tokens, s.reserved_tokens, s.evictions) == (2, 6, 8, 1)
    assert c.find_prefix([1, 2, 3, 0]) is not None
    assert c.find_prefix([4, 5, 6, 0]) is None
    assert c.find_prefix([7, 8, 9, 0]) is not None


def test_index_preserves_descendant_entries_after_branch_removal(pc):
    _, c = _cache(pc, 8, 4)
    shorter = _add(c, [1, 2, 3], False, 10)
    _add(c, [1, 2, 3, 4], False, 11)
    c.remove_entry(shorter.index)
    s = c.stats()
    assert (s.entry_count, s.resident_tokens) == (1, 4)
    assert c.find_prefix([1, 2, 3, 0]) is None
    assert not c.contains_prompt_prefix([1, 2, 3, 4, 5], 3)
    assert c.contains_prompt_prefix([1, 2, 3, 4, 5], 4)
    longest = c.find_prefix([1, 2, 3, 4, 5])
    assert longest.len == 4 and c.cached_next_token(longest) == 11


def test_returns_shifted_match_after_extending_and_evicting_earlier_entry(pc):
    pool, c = _cache(pc, 5, 2)
    _add(c, [9, 9], False, 10)
    reuse = _add(c, [1, 2, 3], False, 11)
    assert reuse.index == 1
    work = _work_table(pool, c, reuse, 5)
    stored, _ = c.store_prefix_from_work([1, 2, 3, 4, 5], reuse, work, next_token=12)
    assert (stored.index, stored.len) == (0, 5)
    s = c.stats()
    assert (s.entry_count, s.evictions) == (1, 1)
    assert c.find_prefix([9, 9, 0]) is None
    assert c.find_prefix([1, 2, 3, 4, 5, 6]) == stored
    # prefixState(.{ index = stored.index, len = reuse.len }): the decode prefix is reuse.len rows
    from peregrine_b200.capi import Match
    pages = c.fork(Match(stored.index, reuse.len))
    assert len(pages) == -(-reuse.len // PAGE)
    pool.release(pages)


def test_preserves_pinned_entries_across_eviction(pc):
    _, c = _cache(pc, 8, 4)
    _add(c, [1, 2, 3], True, 10)
    _add(c, [4, 5, 6], False, 11)
    _add(c, [7, 8, 9], False, 12)
    s = c.stats()
    assert (s.entry_count, s.resident_tokens, s.reserved_tokens, s.pinned_count) == (2, 6, 8, 1)
    assert c.find_prefix([1, 2, 3, 0]) is not None
    assert c.find_prefix([4, 5, 6, 0]) is None
    assert c.find_prefix([7, 8, 9, 0]) is not None


def test_store_marks_hidden_valid_for_fresh_entry_with_real_hiddens(pc):
    pool, c = _cache(pc, 8, 4)
    c.enable_hidden_tracking()
    work = _work_table(pool, c, None, 3)
    m, copy_linear = c.store_prefix_from_work([1, 2, 3], None, work, suffix_hidden=True)
    assert c.entry_hidden_valid(m) and copy_linear
    # the entry adopted the work sequence's pages: its hidden rows are the ones written there
    assert np.array_equal(c.entry_pages(m), work)


def test_store_preserves_reused_hidden_rows_and_extends_validity(pc):
    pool, c = _cache(pc, 16, 4)
    c.enable_hidden_tracking()
    a, _ = c.store_prefix_from_work([1, 2, 3], None, _work_table(pool, c, None, 3),
                                    suffix_hidden=True)
    assert c.entry_hidden_valid(a)
    work = _work_table(pool, c, a, 5)
    b, copy_linear = c.store_prefix_from_work([1, 2, 3, 4, 5], a, work, suffix_hidden=True)
    assert c.entry_hidden_valid(b) and copy_linear


def test_store_clears_hidden_valid_when_suffix_hiddens_are_absent(pc):
    pool, c = _cache(pc, 16, 4)
    c.enable_hidden_tracking()
    a, _ = c.store_prefix_from_work([1, 2, 3], None, _work_table(pool, c, None, 3),
                                    suffix_hidden=True)
    assert c.entry_hidden_valid(a)
    b, _ = c.store_prefix_from_work([1, 2, 3, 4, 5], a, _work_table(pool, c, a, 5),
                                    suffix_hidden=False)
    assert not c.entry_hidden_valid(b)


def test_store_reads_reuse_validity_from_the_shifted_entry(pc):
    pool, c = _cache(pc, 8, 4)
    c.enable_hidden_tracking()
    a, _ = c.store_prefix_from_work([1, 2, 3], None, _work_table(pool, c, None, 3),
                                    suffix_hidden=True)
    assert a.index == 0 and c.entry_hidden_valid(a)
    b, _ = c.store_prefix_from_work([4, 5, 6], None, _work_table(pool, c, None, 3),
                                    suffix_hidden=True)
    assert b.index == 1 and c.entry_hidden_valid(b)
    assert c.stats().reserved_tokens == 8
    work = _work_table(pool, c, b, 5)
    m, _ = c.store_prefix_from_work([4, 5, 6, 7, 8], b, work, suffix_hidden=True)
    assert c.entry_count() == 1 and m.index == 0
    assert c.entry_hidden_valid(m)
    # the reused rows 0..3 are B's: the entry's first page is the work page copied from B's
    assert np.array_equal(c.entry_pages(m), work)


def test_stats_track_token_level_hit_ratio(pc):
    _, c = _cache(pc, 4096, 1600)
    c.record_miss()
    c.record_computed_tokens(1000)
    a = c.start_direct_entry([1] * 1000)
    c.finish_loaded_entry(a)
    c.record_hit(800)
    c.record_computed_tokens(400)
    c.record_hit(1000)
    c.record_computed_tokens(0)
    s = c.stats()
    assert (s.hits, s.misses, s.hit_tokens, s.computed_tokens) == (2, 1, 1800, 1400)
    assert abs(s.hit_tokens / (s.hit_tokens + s.computed_tokens) - 0.5625) < 1e-9


# ------------------------------------------------------------------------ page-sharing contract

def test_page_pool_refcounts_and_copy_on_write(pc):
    from peregrine_b200.capi import PgcError
    pool = pc.PagePool(8)
    a = pool.alloc(3)
    assert list(a) == [0, 1, 2] and pool.free_pages == 5
    with pytest.raises(PgcError, match="CAPACITY"):
        pool.alloc(6)
    assert pool.free_pages == 5  # nothing taken
    pool.retain(a[:2])
    assert [pool.refcount(int(p)) for p in a] == [2, 2, 1]
    t = a.copy()
    assert pool.make_writable(t, 2) == (2, 2)  # sole holder: no copy
    src, dst = pool.make_writable(t, 0)  # shared: fresh page, our reference moves to it
    assert src == 0 and dst not in a and t[0] == dst
    assert pool.refcount(0) == 1 and pool.refcount(dst) == 1
    pool.release(t)
    pool.release(a[:2])
    assert pool.free_pages == 8
    with pytest.raises(PgcError, match="BOUNDS"):
        pool.release([0])  # already free
    b = pool.alloc(1)
    with pytest.raises(PgcError, match="BOUNDS"):
        pool.release([int(b[0]), int(b[0])])  # one reference, listed twice
    with pytest.raises(PgcError, match="BOUNDS"):
        pool.retain([99])


def test_fork_shares_pages_and_eviction_frees_only_unheld_pages(pc):
    pool, c = _cache(pc, 1000, 16, pages=16)
    m = c.start_direct_entry(list(range(40)))  # 3 pages, the last one partial
    c.finish_direct_entry(m, 7)
    entry_pages = c.entry_pages(m)
    assert pool.free_pages == 13
    hit = c.find_prefix(list(range(40)) + [99, 98])
    assert hit == m
    table = c.fork(hit)
    assert np.array_equal(table, entry_pages)
    assert all(pool.refcount(int(p)) == 2 for p in table)
    src, dst = pool.make_writable(table, 2)  # the request will append at position 40
    assert src == entry_pages[2] and pool.refcount(int(src)) == 1
    c.remove_entry(m.index)  # entry gone: its unshared page is freed, the forked two stay
    assert pool.refcount(int(entry_pages[0])) == 1 and pool.refcount(int(entry_pages[2])) == 0
    assert pool.free_pages == 16 - 3
    pool.release(table)
    assert pool.free_pages == 16


def test_start_direct_and_load_slot_evict_for_pages(pc):
    from peregrine_b200.capi import PgcError
    pool, c = _cache(pc, 10_000, 16, pages=8)
    a = c.start_direct_entry(list(range(64)))  # 4 pages
    c.finish_direct_entry(a, 1)
    b = c.start_direct_entry(list(range(100, 164)))  # needs the last 4 pages
    c.finish_direct_entry(b, 2)
    assert pool.free_pages == 0
    held = c.fork(c.find_prefix(list(range(100, 164))))  # a running sequence holds b's pages
    c.start_direct_entry(list(range(200, 232)))  # 2 pages: evicts the LRU entry (a)
    s = c.stats()
    assert s.evictions == 1 and c.find_prefix(list(range(64))) is None
    with pytest.raises(PgcError, match="CAPACITY"):
        c.evict_for_pages(8)  # everything evicted, b's pages are still held by the sequence
    assert c.entry_count() == 0 and pool.free_pages == 4
    pool.release(held)
    m = c.load_entry_slot(list(range(50)))
    assert c.find_prefix(list(range(50))) is None  # indexed only by finish_loaded_entry
    c.finish_loaded_entry(m)
    assert c.find_prefix(list(range(51))) == m
    assert c.persisted_entry() == m and c.pinned_entry_count() == 1


@pytest.mark.parametrize("seed", [5, 6, 7])
def test_random_walk_keeps_bookkeeping_consistent(pc, seed):
    """Seeded random operations; after each: every page's refcount equals its holders (entries
    + live sequences), free pages complement the held ones, reserved tokens equal the sum of
    entry capacities and stay within the budget, and every entry is found by its own tokens."""
    from peregrine_b200.capi import PgcError
    rng = np.random.default_rng(seed)
    npages = 96
    pool, c = _cache(pc, 600, 48, pages=npages, slots=6)
    bases = [list(rng.integers(0, 50, 100)) for _ in range(3)]
    seqs = []  # live request tables
    stores = reuses = 0
    for step in range(600):
        op = rng.integers(0, 5)
        # prompts extend one of a few shared prefixes, so hits, forks and in-place extension
        # of entries are frequent
        base = bases[rng.integers(0, 3)]
        tail = rng.integers(0, 20) if rng.random() < 0.3 else 0
        prompt = base[:rng.integers(1, 100)] + list(rng.integers(0, 50, tail))
        try:
            if op == 0:
                m = c.start_direct_entry(prompt, pinned=bool(rng.random() < 0.1))
                c.finish_direct_entry(m, 1)
            elif op in (1, 2):
                hit = c.find_prefix(prompt)
                if hit is not None and hit.len == len(prompt):
                    continue
                need = -(-len(prompt) // PAGE)
                c.evict_for_pages(need)
                hit = c.find_prefix(prompt)
                table = _work_table(pool, c, hit, len(prompt))
                m, _ = c.store_prefix_from_work(prompt, hit, table)
                stores += 1
                reuses += hit is not None
                if op == 2 and len(seqs) < 4:
                    seqs.append(table)
                else:
                    pool.release(table)
            elif op == 3 and seqs:
                pool.release(seqs.pop(int(rng.integers(0, len(seqs)))))
            elif op == 4 and c.entry_count():
                c.remove_entry(int(rng.integers(0, c.entry_count())))
        except PgcError as e:
            assert e.status in (-2, -11), e
        holders = np.zeros(npages, np.int64)
        s = c.stats()
        cap = 0
        for i in range(s.entry_count):
            info, toks, pages = c.entry(i)
            np.add.at(holders, pages, 1)
            cap += info.capacity
            assert len(pages) == -(-len(toks) // PAGE)
            f = c.find_prefix(toks)
            assert f is not None and f.index == i and f.len == len(toks)
        for t in seqs:
            np.add.at(holders, t, 1)
        refs = np.array([pool.refcount(p) for p in range(npages)])
        assert np.array_equal(refs, holders), step
        assert pool.free_pages == int((refs == 0).sum())
        assert s.reserved_tokens == cap <= 600
    assert stores > 100 and reuses > 50 and c.stats().evictions > 20
    # the path-compressed index holds at most two nodes per entry, and only the root when empty
    assert c.stats().trie_nodes <= 2 * c.entry_count() + 1
    for i in reversed(range(c.entry_count())):
        c.remove_entry(i)
    assert c.stats().trie_nodes == 1
    for t in seqs:
        pool.release(t)
    assert pool.free_pages == npages


def test_index_splits_and_folds_runs(pc):
    """Split an edge (a shorter prefix, a branch), then remove entries so that nodes fold back;
    every remaining entry is still found with its own length."""
    _, c = _cache(pc, 10_000, 16)
    long_ = list(range(100))
    _add(c, long_, False, 1)
    assert c.stats().trie_nodes == 2
    _add(c, long_[:50], False, 2)        # split at 50
    _add(c, long_[:50] + [7, 7], False, 3)  # branch at 50
    _add(c, long_[:25], False, 4)        # split at 25
    assert c.stats().trie_nodes == 5
    assert c.find_prefix(long_ + [1]).len == 100
    assert c.find_prefix(long_[:60]).len == 50
    assert c.find_prefix(long_[:50] + [7, 7, 7]).len == 52
    assert c.find_prefix(long_[:30]).len == 25
    assert c.find_prefix(long_[:24]) is None
    c.remove_entry(c.find_prefix(long_[:50]).index)  # node at 50 keeps two children
    assert c.stats().trie_nodes == 5 and c.find_prefix(long_[:60]).len == 25
    c.remove_entry(c.find_prefix(long_[:50] + [7, 7]).index)  # 50 folds into the long leaf
    assert c.stats().trie_nodes == 3
    assert c.find_prefix(long_ + [1]).len == 100 and c.find_prefix(long_[:60]).len == 25
    c.remove_entry(c.find_prefix(long_[:30]).index)  # 25 folds too
    assert c.stats().trie_nodes == 2 and c.find_prefix(long_).len == 100


# ------------------------------------------------------------------------------------- GPU

@pytest.mark.gpu
def test_forked_requests_share_prefix_pages_on_gpu(cuda, oracle, pc):
    """Entry of 40 tokens (3 pages, last partial). Requests B and C fork it, copy the partial
    page on write (one pgc_copy_regions launch over the K and V pools of two layers) and write
    different suffixes at positions 40..; B, C and the entry then snapshot bit-exact to their
    logical rows and decode within tolerance of the oracle."""
    import torch

    from _util import assert_attn_close, dev, host_u16
    from peregrine_b200 import capi
    rng = np.random.default_rng(11)
    npages, layers = 32, 2
    pool, c = _cache(pc, 4096, 16, pages=npages)
    pools = [torch.zeros((npages, NKV, PAGE, D), dtype=torch.int16, device="cuda")
             for _ in range(2 * layers)]

    def rows(n, seed):
        return oracle.normal_bf16(n * NKV * D, seed).reshape(n, NKV, D)

    def write(table, start, k, v, layer):
        n = k.shape[0]
        kd = dev(np.ascontiguousarray(k.transpose(1, 0, 2)))        # [4][n][256]
        vd = dev(np.ascontiguousarray(v.transpose(1, 2, 0)))        # [4][256][n]
        t = dev(table.reshape(1, -1))
        capi.kv_restore_dense(kd, vd, n, 0, pools[2 * layer], pools[2 * layer + 1], t, start, n)
        torch.cuda.synchronize()

    def read(table, n, layer):
        t = dev(table.reshape(1, -1))
        kd = torch.zeros((NKV, n, D), dtype=torch.int16, device="cuda")
        vd = torch.zeros((NKV, D, n), dtype=torch.int16, device="cuda")
        capi.kv_snapshot_dense(pools[2 * layer], pools[2 * layer + 1], t, 0, kd, vd, n, 0, n)
        torch.cuda.synchronize()
        return host_u16(kd).transpose(1, 0, 2), host_u16(vd).transpose(2, 0, 1)

    prompt_a = list(range(1000, 1040))
    ka = [rows(40, 10 + l) for l in range(layers)]
    va = [rows(40, 20 + l) for l in range(layers)]
    m = c.start_direct_entry(prompt_a)
    ta = c.entry_pages(m)
    for l in range(layers):
        write(ta, 0, ka[l], va[l], l)
    c.finish_direct_entry(m, 5)

    suffix = {}
    tables = {}
    for name, seed, n_new in (("B", 30, 30), ("C", 40, 9)):
        hit = c.find_prefix(prompt_a + [7] * n_new)
        assert hit is not None and hit.len == 40
        table = c.fork(hit)
        src, dst = pool.make_writable(table, 2)
        assert src != dst
        pc.copy_page(pools, src, dst)
        extra = -(-(40 + n_new) // PAGE) - len(table)
        table = np.concatenate([table, pool.alloc(extra)]).astype(np.int32)
        ks = [rows(n_new, seed + l) for l in range(layers)]
        vs = [rows(n_new, seed + 5 + l) for l in range(layers)]
        for l in range(layers):
            write(table, 40, ks[l], vs[l], l)
        suffix[name] = (ks, vs)
        tables[name] = table
    torch.cuda.synchronize()

    q = oracle.normal_bf16(16 * D, 3).reshape(1, 1, 16, D)
    for name in ("A", "B", "C"):
        for l in range(layers):
            if name == "A":
                k_all, v_all, table = ka[l], va[l], ta
            else:
                ks, vs = suffix[name]
                k_all = np.concatenate([ka[l], ks[l]])
                v_all = np.concatenate([va[l], vs[l]])
                table = tables[name]
            n = k_all.shape[0]
            kr, vr = read(table, n, l)
            assert np.array_equal(kr, k_all) and np.array_equal(vr, v_all), (name, l)
            kp = host_u16(pools[2 * l])
            vp = host_u16(pools[2 * l + 1])
            t2 = table.reshape(1, -1)
            ref, _ = oracle.decode_paged(q, kp, vp, t2, np.array([n], np.int32), 1 / 16)
            out = torch.empty((1, 1, 16, D), dtype=torch.int16, device="cuda")
            ws = torch.empty(capi.decode_workspace_bytes(1, 1, n), dtype=torch.uint8, device="cuda")
            capi.decode_attn(dev(q), pools[2 * l], pools[2 * l + 1], dev(t2),
                             dev(np.array([n], np.int32)), n, 1 / 16, out, ws)
            torch.cuda.synchronize()
            assert_attn_close(host_u16(out)[0, 0], ref[0, 0])
