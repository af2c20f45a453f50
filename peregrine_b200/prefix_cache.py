"""Page pool and page-refcounted prompt-prefix cache: Python face of the native cache in
csrc/prefix_cache.cpp (C ABI in include/peregrine_cuda.h).

Method names follow the reference cache (src/server/prefix_state_cache.zig: findPrefix,
containsPromptPrefix, touch, recordHit, startDirectEntry, storePrefixFromWork, removeEntry,
loadEntrySlot, ...), so a caller of the reference reads the same flow. The difference is what an
entry holds: page ids in the shared KV/hidden pools instead of a private model state, so a hit
forks pages (refcount) and only the partial page at the end of a match is copied, on the device,
before the request writes into it (`copy_page`).

All bookkeeping runs in the native library; nothing here computes.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import capi
from .capi import Match, PrefixEntry, PrefixStats, check, lib


def _u32(tokens) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))


class PagePool:
    """Refcounted page ids [0, num_pages) of the per-layer page pools."""

    def __init__(self, num_pages: int):
        self._h = lib().pgc_page_pool_create(num_pages)
        if not self._h:
            raise capi.PgcError(capi.STATUS_INVALID, "pgc_page_pool_create")
        self.num_pages = num_pages

    def close(self) -> None:
        if self._h:
            lib().pgc_page_pool_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def handle(self):
        return self._h

    def alloc(self, n: int) -> np.ndarray:
        out = np.empty(n, np.int32)
        check(lib().pgc_page_pool_alloc(self._h, n, out.ctypes.data), "pgc_page_pool_alloc")
        return out

    def retain(self, pages) -> None:
        p = np.ascontiguousarray(pages, dtype=np.int32)
        check(lib().pgc_page_pool_retain(self._h, p.ctypes.data, p.size), "pgc_page_pool_retain")

    def release(self, pages) -> None:
        p = np.ascontiguousarray(pages, dtype=np.int32)
        check(lib().pgc_page_pool_release(self._h, p.ctypes.data, p.size), "pgc_page_pool_release")

    def refcount(self, page: int) -> int:
        r = lib().pgc_page_pool_refcount(self._h, page)
        if r < 0:
            raise capi.PgcError(r, "pgc_page_pool_refcount")
        return r

    @property
    def free_pages(self) -> int:
        return lib().pgc_page_pool_free_pages(self._h)

    def make_writable(self, table: np.ndarray, slot: int) -> tuple[int, int]:
        """Copy-on-write of table[slot] (int32 array, updated in place); returns (src, dst)
        page ids, equal when nothing has to be copied."""
        assert table.dtype == np.int32 and table.flags.c_contiguous
        src, dst = C.c_int32(), C.c_int32()
        check(lib().pgc_page_pool_make_writable(self._h, table.ctypes.data, slot, C.byref(src),
                                                C.byref(dst)), "pgc_page_pool_make_writable")
        return src.value, dst.value


def copy_page(pools, src: int, dst: int, stream=None) -> None:
    """Device copy of page `src` to page `dst` in every per-page pool tensor of `pools` (K and
    V of each full layer, the hidden-row pool, ...): one pgc_copy_regions launch."""
    if src == dst:
        return
    pairs = []
    for t in pools:
        page_bytes = t[0].numel() * t.element_size()
        base = t.data_ptr()
        pairs.append((base + dst * page_bytes, base + src * page_bytes, page_bytes))
    for i in range(0, len(pairs), capi.MAX_REGIONS):
        capi.copy_regions(pairs[i:i + capi.MAX_REGIONS], stream=stream)


class PrefixCache:
    """The reference's resident prefix cache (Cache, prefix_state_cache.zig:292-567) over a
    PagePool. A Match stays valid only until the next mutating call, as in the reference."""

    def __init__(self, pool: PagePool, max_cache_tokens: int, prefill_chunk_tokens: int,
                 state_slots: int = 64, page_tokens: int = capi.PAGE_TOKENS):
        self.pool = pool
        self.page_tokens = page_tokens
        self._h = lib().pgc_prefix_cache_create(pool.handle, page_tokens, max_cache_tokens,
                                                prefill_chunk_tokens, state_slots)
        if not self._h:
            raise capi.PgcError(capi.STATUS_INVALID, "pgc_prefix_cache_create")

    def close(self) -> None:
        if self._h:
            lib().pgc_prefix_cache_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    # -- lookups
    def find_prefix(self, prompt) -> Match | None:
        p = _u32(prompt)
        m = Match()
        r = lib().pgc_prefix_cache_find(self._h, p.ctypes.data, p.size, C.byref(m))
        if r < 0:
            raise capi.PgcError(r, "pgc_prefix_cache_find")
        return m if r == 1 else None

    def contains_prompt_prefix(self, prompt, prefix_len: int) -> bool:
        p = _u32(prompt)
        r = lib().pgc_prefix_cache_contains(self._h, p.ctypes.data, p.size, prefix_len)
        if r < 0:
            raise capi.PgcError(r, "pgc_prefix_cache_contains")
        return r == 1

    def stats(self) -> PrefixStats:
        s = PrefixStats()
        check(lib().pgc_prefix_cache_stats(self._h, C.byref(s)), "pgc_prefix_cache_stats")
        return s

    def entry_count(self) -> int:
        return self.stats().entry_count

    def pinned_entry_count(self) -> int:
        return self.stats().pinned_count

    def entry(self, index: int) -> tuple[PrefixEntry, np.ndarray, np.ndarray]:
        info = PrefixEntry()
        check(lib().pgc_prefix_cache_entry(self._h, index, C.byref(info), None, 0, None, 0),
              "pgc_prefix_cache_entry")
        toks = np.empty(info.token_count, np.uint32)
        pages = np.empty(info.page_count, np.int32)
        check(lib().pgc_prefix_cache_entry(self._h, index, C.byref(info), toks.ctypes.data,
                                           toks.size, pages.ctypes.data, pages.size),
              "pgc_prefix_cache_entry")
        return info, toks, pages

    def cached_next_token_valid(self, m: Match) -> bool:
        return bool(self.entry(m.index)[0].next_token_valid)

    def cached_next_token(self, m: Match) -> int:
        return self.entry(m.index)[0].next_token

    def entry_hidden_valid(self, m: Match) -> bool:
        if m.index < 0 or m.index >= self.entry_count():
            return False
        return bool(self.entry(m.index)[0].hidden_valid)

    def entry_pages(self, m: Match) -> np.ndarray:
        return self.entry(m.index)[2]

    def persisted_entry(self) -> Match | None:
        m = Match()
        r = lib().pgc_prefix_cache_persisted(self._h, C.byref(m))
        return m if r == 1 else None

    # -- bookkeeping
    def touch(self, m: Match) -> None:
        lib().pgc_prefix_cache_touch(self._h, m)

    def record_hit(self, reused_tokens: int) -> None:
        lib().pgc_prefix_cache_record_hit(self._h, reused_tokens)

    def record_miss(self) -> None:
        lib().pgc_prefix_cache_record_miss(self._h)

    def record_computed_tokens(self, tokens: int) -> None:
        lib().pgc_prefix_cache_record_computed(self._h, tokens)

    def enable_hidden_tracking(self) -> None:
        lib().pgc_prefix_cache_enable_hidden_tracking(self._h)

    def clear_all(self) -> None:
        lib().pgc_prefix_cache_clear_all(self._h)

    # -- mutations
    def remove_entry(self, index: int) -> None:
        check(lib().pgc_prefix_cache_remove(self._h, index), "pgc_prefix_cache_remove")

    def start_direct_entry(self, prefix_ids, pinned: bool = False) -> Match:
        p = _u32(prefix_ids)
        m = Match()
        check(lib().pgc_prefix_cache_start_direct(self._h, p.ctypes.data, p.size, int(pinned),
                                                  C.byref(m)), "pgc_prefix_cache_start_direct")
        return m

    def finish_direct_entry(self, m: Match, next_token: int) -> None:
        check(lib().pgc_prefix_cache_finish_direct(self._h, m, next_token),
              "pgc_prefix_cache_finish_direct")

    def set_entry_hidden_valid(self, m: Match, valid: bool = True) -> None:
        check(lib().pgc_prefix_cache_set_hidden_valid(self._h, m, int(valid)),
              "pgc_prefix_cache_set_hidden_valid")

    def store_prefix_from_work(self, prefix_ids, reuse: Match | None, work_table,
                               suffix_hidden: bool = False, next_token: int | None = None,
                               pinned: bool = False) -> tuple[Match, bool]:
        """Returns (match, copy_linear_state)."""
        p = _u32(prefix_ids)
        t = np.ascontiguousarray(work_table, dtype=np.int32)
        out = Match()
        nt = C.c_uint32(next_token) if next_token is not None else None
        copy_lin = C.c_int(0)
        check(lib().pgc_prefix_cache_store(
            self._h, p.ctypes.data, p.size, C.byref(reuse) if reuse is not None else None,
            t.ctypes.data, t.size, int(suffix_hidden), C.byref(nt) if nt is not None else None,
            int(pinned), C.byref(out), C.byref(copy_lin)), "pgc_prefix_cache_store")
        return out, bool(copy_lin.value)

    def fork(self, m: Match, table_cap: int | None = None) -> np.ndarray:
        """The request's leading block-table pages for m.len tokens (references taken)."""
        cap = table_cap or (m.len + self.page_tokens - 1) // self.page_tokens
        out = np.empty(cap, np.int32)
        n = C.c_int64()
        check(lib().pgc_prefix_cache_fork(self._h, m, out.ctypes.data, cap, C.byref(n)),
              "pgc_prefix_cache_fork")
        return out[:n.value]

    def evict_for_pages(self, need_free: int) -> None:
        check(lib().pgc_prefix_cache_evict_for_pages(self._h, need_free),
              "pgc_prefix_cache_evict_for_pages")

    def load_entry_slot(self, token_ids) -> Match:
        p = _u32(token_ids)
        m = Match()
        check(lib().pgc_prefix_cache_load_slot(self._h, p.ctypes.data, p.size, C.byref(m)),
              "pgc_prefix_cache_load_slot")
        return m

    def finish_loaded_entry(self, m: Match) -> None:
        check(lib().pgc_prefix_cache_finish_loaded(self._h, m), "pgc_prefix_cache_finish_loaded")
