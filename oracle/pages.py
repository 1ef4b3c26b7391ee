"""CPU restatement of the device page allocator (TEST INFRASTRUCTURE ONLY).

The reference has no paged cache (its KV cache is dense per slot,
src/climbing_gym/inference/lfm25_engine.py:1187-1221), so this oracle pins *this* engine's
allocator: a pure integer function of the reserve / step / release / fork trace. Rules:
pages are handed out lowest id first; within one call entries are served in entry order and a
slot's new blocks in ascending block order; a page returns to the pool when its reference
count reaches zero. parity unpinned against the reference (nothing to pin to); the slot-level
bookkeeping it sits under is pinned by tests/golden/kernels.json ``record_sample``.
"""
from __future__ import annotations

import numpy as np


class PagePoolOracle:
    def __init__(self, n_pages: int, page_size: int, max_blocks: int, n_slots: int):
        self.n_pages, self.page_size, self.max_blocks, self.n_slots = n_pages, page_size, max_blocks, n_slots
        self.free = np.ones(n_pages, bool)
        self.refcount = np.zeros(n_pages, np.int32)
        self.block_table = np.full((n_slots, max_blocks), -1, np.int32)
        self.n_blocks = np.zeros(n_slots, np.int32)
        self.seq_lens = np.zeros(n_slots, np.int32)
        self.status = 0

    def reserve(self, slot_ids, need_tokens):
        for slot, need in zip(slot_ids, need_tokens):
            if slot < 0 or slot >= self.n_slots:
                continue
            target = -(-int(need) // self.page_size)
            if target > self.max_blocks:
                self.status |= 8
                target = self.max_blocks
            while self.n_blocks[slot] < target:
                free = np.flatnonzero(self.free)
                if free.size == 0:
                    self.status |= 1
                    break
                page = int(free[0])
                self.free[page] = False
                self.refcount[page] = 1
                self.block_table[slot, self.n_blocks[slot]] = page
                self.n_blocks[slot] += 1

    def step(self, active, slots=None):
        rows = range(len(active))
        ids = [(int(slots[r]) if slots is not None else r) for r in rows if active[r]]
        ids = [s for s in ids if s >= 0]
        self.reserve(ids, [int(self.seq_lens[s]) + 1 for s in ids])

    def release(self, mask):
        for slot in np.flatnonzero(np.asarray(mask)):
            for b in range(int(self.n_blocks[slot])):
                page = int(self.block_table[slot, b])
                self.block_table[slot, b] = -1
                if page >= 0:
                    self.refcount[page] -= 1
                    if self.refcount[page] == 0:
                        self.free[page] = True
            self.n_blocks[slot] = 0
            self.seq_lens[slot] = 0

    def fork(self, src_slots, dst_slots, prefix_lens):
        for src, dst, length in zip(src_slots, dst_slots, prefix_lens):
            full = int(length) // self.page_size
            for b in range(full):
                page = int(self.block_table[src, b])
                self.block_table[dst, b] = page
                self.refcount[page] += 1
            self.n_blocks[dst] = full
        self.reserve(dst_slots, prefix_lens)
        for dst, length in zip(dst_slots, prefix_lens):
            self.seq_lens[dst] = length

    def bitmap_words(self) -> np.ndarray:
        words = np.zeros(-(-self.n_pages // 32), np.uint32)
        for page in np.flatnonzero(self.free):
            words[page >> 5] |= np.uint32(1 << (page & 31))
        return words
