"""CPU oracle of the copy-on-write page transaction.

TEST INFRASTRUCTURE ONLY. A direct, sequential restatement of the reference's
PagedTreeCache (python/branchcraft_torch/transaction.py:30-150) over numpy
arrays: K/V pools [P, 16, Hkv, D] of FP16 bit patterns, a refcounted free list
that starts as [P-1, ..., 0] and pops from the end, fork / checkpoint /
rollback / accept, and commit, which clones a shared partial last page
(copying the whole page) before writing the accepted path node by node.
"""
from __future__ import annotations

import numpy as np


class CowOracle:
    def __init__(self, physical_pages, kv_heads, head_dim):
        self.k = np.zeros((physical_pages, 16, kv_heads, head_dim), np.uint16)
        self.v = np.zeros_like(self.k)
        self.refcount = [0] * physical_pages          # transaction.py:31
        self.free = list(range(physical_pages - 1, -1, -1))  # :32
        self.pages = {}
        self.lengths = {}
        self._next = 0

    def _alloc(self):                                  # :37-43
        if not self.free:
            raise RuntimeError("KV page pool exhausted")
        page = self.free.pop()
        assert self.refcount[page] == 0
        self.refcount[page] = 1
        return page

    def _release(self, page):                          # :45-48
        self.refcount[page] -= 1
        if self.refcount[page] == 0:
            self.free.append(page)

    def new(self, prefix_k, prefix_v):                 # :50-71
        n = prefix_k.shape[0]
        count = (n + 15) // 16
        if len(self.free) < count:
            raise RuntimeError("KV page pool exhausted")
        r = self._next
        self._next += 1
        self.pages[r] = []
        self.lengths[r] = n
        for start in range(0, n, 16):
            page = self._alloc()
            self.pages[r].append(page)
            m = min(16, n - start)
            self.k[page, :m] = prefix_k[start:start + m]
            self.v[page, :m] = prefix_v[start:start + m]
        return r

    def fork(self, source):                            # :73-80
        r = self._next
        self._next += 1
        self.pages[r] = list(self.pages[source])
        self.lengths[r] = self.lengths[source]
        for page in self.pages[r]:
            self.refcount[page] += 1
        return r

    def checkpoint(self, r):                           # :82-86
        pages = list(self.pages[r])
        for page in pages:
            self.refcount[page] += 1
        return {"request": r, "pages": pages, "length": self.lengths[r], "active": True}

    def rollback(self, snap):                          # :88-95
        if not snap["active"]:
            raise RuntimeError("snapshot already consumed")
        for page in self.pages[snap["request"]]:
            self._release(page)
        self.pages[snap["request"]] = snap["pages"]
        self.lengths[snap["request"]] = snap["length"]
        snap["active"] = False

    def accept(self, snap):                            # :97-102
        if not snap["active"]:
            raise RuntimeError("snapshot already consumed")
        for page in snap["pages"]:
            self._release(page)
        snap["active"] = False

    def commit(self, r, path, draft_k, draft_v):       # :114-150
        """draft_k/draft_v: [N, Hkv, D] uint16 for this request."""
        if not path or len(path) > draft_k.shape[0]:
            raise ValueError("path is empty or longer than draft")
        if any(n < 0 or n >= draft_k.shape[0] for n in path):
            raise ValueError("path node out of range")
        old_length = self.lengths[r]
        old_pages = self.pages[r]
        new_count = (old_length + len(path) + 15) // 16
        copy_partial = old_length % 16 != 0 and self.refcount[old_pages[-1]] > 1
        needed = new_count - len(old_pages) + int(copy_partial)
        if len(self.free) < needed:
            raise RuntimeError("KV page pool exhausted")
        if copy_partial:
            old = old_pages[-1]
            fresh = self._alloc()
            self.k[fresh] = self.k[old]
            self.v[fresh] = self.v[old]
            old_pages[-1] = fresh
            self._release(old)
        while len(old_pages) < new_count:
            old_pages.append(self._alloc())
        for i, node in enumerate(path):
            pos = old_length + i
            self.k[old_pages[pos // 16], pos % 16] = draft_k[node]
            self.v[old_pages[pos // 16], pos % 16] = draft_v[node]
        self.lengths[r] += len(path)
