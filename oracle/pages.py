"""CPU model of the paged K/V window: page allocator, page table, append and
window gather.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The reference keeps one dense window per slot and moves it with a shift
(``parakeet/modules/cache.py:36-45``) plus ``index_select``/``index_copy_``
(``parakeet/engine/scheduler.py:128-201``).  The CUDA path keeps the same
window in fixed-size pages instead.  This model is the specification the
device allocator must match op for op; its page-id values have no reference
counterpart ("parity unpinned by the reference" for ids), while the window
it gathers is pinned bit-exactly against the reference's dense window.

Frame slots.  Each step writes T = right + 1 rows per stream whatever the
chunk's valid ``length`` is, exactly like the reference's shift-by-T.  A
stream that has written ``w`` rows before a step sees window rows
j = 0 .. left + T - 1 at absolute slot a = w - left + j; a < 0 reads zeros
(the reference zeroes a slot on acquire).  Slot a lives in logical page
a // page_size, stored in page-table ring entry (a // page_size) % ring.

Step order (every step, one batch):
  0. releases: pages of finished streams, in release order, to the free tail
  1. frees:  per batch row in batch order, logical pages n with
             (n + 1) * page_size <= w - left (wholly left of the window)
  2. allocs: per batch row in batch order, pages n up to (w + T - 1) // ps
             popped from the free head
  3. the layers append rows [w, w + T) and read rows [w - left, w + T)
  4. end: w += T, processed += length, cache_len = min(cache_len + length, left)
"""
from __future__ import annotations

from collections import deque

import numpy as np


def pages_per_stream(left, chunk, page_size):
    """Most logical pages one stream's window [w - left, w + chunk) can touch."""
    span = left + chunk - 1
    return -(-span // page_size) + 1


def ring_size(left, chunk, page_size):
    n = pages_per_stream(left, chunk, page_size)
    r = 1
    while r < n:
        r *= 2
    return r


class PagePoolModel:
    """FIFO page free list + per-slot page-table ring + per-slot counters."""

    def __init__(self, num_pages, num_slots, left, chunk, page_size=16,
                 init_order=None):
        self.num_pages = num_pages
        self.left, self.chunk, self.ps = left, chunk, page_size
        self.ring = ring_size(left, chunk, page_size)
        order = range(num_pages) if init_order is None else [int(p) for p in init_order]
        self.free = deque(order)
        self.table = np.full((num_slots, self.ring), -1, np.int32)
        self.first = np.zeros(num_slots, np.int64)     # oldest logical page held
        self.next = np.zeros(num_slots, np.int64)      # next logical page to allocate
        self.written = np.zeros(num_slots, np.int64)   # rows written (T per step)
        self.processed = np.zeros(num_slots, np.int64)
        self.cache_len = np.zeros(num_slots, np.int64)
        self.pending_release: list[int] = []
        self.error = 0

    # host side: a slot leaves; its pages return at the start of the next step
    def release_slot(self, slot):
        self.pending_release.append(int(slot))

    def _drop_pages(self, slot):
        for n in range(self.first[slot], self.next[slot]):
            e = n % self.ring
            self.free.append(int(self.table[slot, e]))
            self.table[slot, e] = -1
        self.first[slot] = self.next[slot] = 0
        self.written[slot] = self.processed[slot] = self.cache_len[slot] = 0

    def begin_step(self, slots):
        for s in self.pending_release:                                  # 0
            self._drop_pages(s)
        self.pending_release = []
        for s in slots:                                                 # 1
            w = self.written[s]
            while self.first[s] < self.next[s] and \
                    (self.first[s] + 1) * self.ps <= w - self.left:
                e = self.first[s] % self.ring
                self.free.append(int(self.table[s, e]))
                self.table[s, e] = -1
                self.first[s] += 1
        need = []
        for s in slots:                                                 # 2
            last = (self.written[s] + self.chunk - 1) // self.ps
            need.append(max(0, int(last - self.next[s] + 1)))
        if sum(need) > len(self.free):
            self.error = 1
            return False
        for s, n in zip(slots, need):
            for _ in range(n):
                self.table[s, self.next[s] % self.ring] = self.free.popleft()
                self.next[s] += 1
        return True

    def end_step(self, slots, lengths):
        for s, n in zip(slots, lengths):                                # 4
            self.written[s] += self.chunk
            self.processed[s] += int(n)
            self.cache_len[s] = min(self.cache_len[s] + int(n), self.left)

    def locate(self, slot, a):
        """(page id, row in page) of absolute slot a, or None for a < 0."""
        if a < 0:
            return None
        return int(self.table[slot, (a // self.ps) % self.ring]), int(a % self.ps)


class PagedKVModel:
    """Page pool contents [pages, L, 2, page_size, D] plus a PagePoolModel."""

    def __init__(self, pool: PagePoolModel, num_layers, dim, dtype=np.float64):
        self.pool = pool
        self.kv = np.zeros((pool.num_pages, num_layers, 2, pool.ps, dim), dtype)

    def append(self, layer, slots, key, value):
        """Write rows [w, w + T) of every batch row (key/value: [B, T, D])."""
        for b, s in enumerate(slots):
            w = self.pool.written[s]
            for t in range(self.pool.chunk):
                pg, r = self.pool.locate(s, w + t)
                self.kv[pg, layer, 0, r] = key[b, t]
                self.kv[pg, layer, 1, r] = value[b, t]

    def gather(self, layer, slots):
        """Materialise the [B, left + T, D] K and V windows of this step."""
        W = self.pool.left + self.pool.chunk
        D = self.kv.shape[-1]
        k = np.zeros((len(slots), W, D), self.kv.dtype)
        v = np.zeros_like(k)
        for b, s in enumerate(slots):
            base = self.pool.written[s] - self.pool.left
            for j in range(W):
                loc = self.pool.locate(s, base + j)
                if loc is not None:
                    k[b, j] = self.kv[loc[0], layer, 0, loc[1]]
                    v[b, j] = self.kv[loc[0], layer, 1, loc[1]]
        return k, v
