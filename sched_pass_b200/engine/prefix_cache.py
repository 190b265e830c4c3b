"""Automatic prefix caching of KV pages.

Requests that share a prompt prefix (a system prompt, a conversation's
history: the shared-prefix structure the trace replay reproduces) reuse the
KV pages of that prefix instead of prefilling it again. The unit is a full
page (``page_size`` tokens): the key of the i-th full block of a prompt is a
chained digest of all tokens up to the end of that block, so equal keys mean
equal prefixes, and the page holding that block's K/V can be shared. Only
full pages are ever shared and a request writes only past its cached prefix,
into pages of its own, so shared pages are read-only and need no copy on
write.

Life of a page: a request's prompt pages are registered once their K/V is
written (after the step that prefilled them commits); a registered page is
referenced by every running request whose block table holds it; when the
last reference goes (the request finished, aborted or was preempted) the page
stays cached but becomes evictable (LRU). The allocator hands out free pages
first and evicts the least recently released cached pages when it runs out.

Every decision depends only on token ids and the step sequence, so all
tensor-parallel ranks keep identical caches.
"""
from __future__ import annotations

import hashlib
from collections import OrderedDict

import numpy as np


def block_keys(tokens: np.ndarray, page_size: int, n_blocks: int) -> list:
    """Chained digests of the first ``n_blocks`` full blocks of ``tokens``."""
    keys, h = [], b"sched-prefix"
    arr = np.asarray(tokens, dtype=np.int32)
    for b in range(n_blocks):
        h = hashlib.blake2b(h + arr[b * page_size:(b + 1) * page_size].tobytes(), digest_size=16).digest()
        keys.append(h)
    return keys


class PrefixCache:
    def __init__(self, page_size: int = 16):
        self.page_size = page_size
        self.page_of: dict = {}      # key -> page
        self.key_of: dict = {}       # page -> key
        self.ref: dict = {}          # page -> requests holding it
        self.idle: OrderedDict = OrderedDict()  # cached pages nobody holds, least recent first
        self.hits = 0                # tokens served from the cache
        self.lookups = 0             # prompt tokens looked up

    @property
    def evictable(self) -> int:
        return len(self.idle)

    def holds(self, page: int) -> bool:
        return page in self.key_of

    def peek(self, tokens: np.ndarray, keys: list | None = None) -> tuple[list, list]:
        """Longest cached prefix of ``tokens`` that leaves at least one token
        to compute (the last prompt token's logits give the first output):
        (its pages, the keys of every full block of ``tokens``). Nothing is
        referenced yet (``acquire``). ``keys``: the block keys of ``tokens``
        if already known (they depend on the tokens only)."""
        n_full = (len(tokens) - 1) // self.page_size
        if keys is None:
            keys = block_keys(tokens, self.page_size, len(tokens) // self.page_size)
        pages = []
        for k in keys[:n_full]:
            p = self.page_of.get(k)
            if p is None:
                break
            pages.append(p)
        return pages, keys

    def acquire(self, pages) -> None:
        """Reference cached pages for one request (they stop being evictable)."""
        for p in pages:
            self.ref[p] = self.ref.get(p, 0) + 1
            self.idle.pop(p, None)

    def register(self, key: bytes, page: int) -> bool:
        """Cache a page the caller holds (its K/V is written). False when
        the key is cached already (under another page, which stays)."""
        if key in self.page_of or page in self.key_of:
            return False
        self.page_of[key] = page
        self.key_of[page] = key
        self.ref[page] = self.ref.get(page, 0) + 1
        return True

    def release(self, page: int) -> None:
        """Drop one reference; the page becomes evictable at zero."""
        n = self.ref[page] - 1
        if n < 0:
            raise ValueError(f"page {page} released more often than held")
        self.ref[page] = n
        if n == 0:
            self.idle[page] = None

    def evict(self, n: int) -> list:
        """Up to ``n`` least recently released pages, forgotten by the cache
        (the caller returns them to the free list)."""
        out = []
        while self.idle and len(out) < n:
            page, _ = self.idle.popitem(last=False)
            key = self.key_of.pop(page)
            del self.page_of[key]
            del self.ref[page]
            out.append(page)
        return out
