"""Host page owner for copy-on-write tree commits.

`PagePool` keeps the reference's page-ownership rules exactly
(python/branchcraft_torch/transaction.py): a refcounted pool whose free list
starts as ``[P-1, ..., 1, 0]`` and hands out pages with ``pop()`` (lowest id
first) and takes them back with ``append`` (transaction.py:32-48); ``fork``
shares every page (:73-80); snapshots pin pages (:82-102); and ``commit``
clones a shared partial last page before writing into it (:114-150).

Unlike the reference, which issues one torch page copy and one kernel launch
per request, ``plan_commit_batch`` replays the same state transitions for a
whole batch of requests on the host and returns ONE plan (page clones, then
per-node writes) that ``bc_commit_batch`` executes in two launches. Running
every clone before every write is equivalent to the sequential order: a clone
only happens when its page is shared (refcount > 1), so no earlier request of
the batch can have written into that page in place, and no page is freed
inside a commit.
"""
from __future__ import annotations

from dataclasses import dataclass, field

PAGE_SIZE = 16


@dataclass
class Snapshot:
    request: int
    pages: list
    length: int
    active: bool = True


@dataclass
class CommitPlan:
    """Flat device-ready arrays (python lists of int)."""

    clone_src: list = field(default_factory=list)
    clone_dst: list = field(default_factory=list)
    entry_request: list = field(default_factory=list)  # index into the draft batch
    entry_node: list = field(default_factory=list)
    entry_page: list = field(default_factory=list)
    entry_slot: list = field(default_factory=list)


class PagePool:
    def __init__(self, physical_pages: int):
        if physical_pages < 1:
            raise ValueError("physical_pages must be positive")
        self.physical_pages = physical_pages
        self.refcount = [0] * physical_pages
        self.free = list(range(physical_pages - 1, -1, -1))
        self.pages: dict[int, list[int]] = {}
        self.lengths: dict[int, int] = {}
        self._next_request = 0

    # -- ownership primitives (transaction.py:37-48)
    def alloc(self) -> int:
        if not self.free:
            raise RuntimeError("KV page pool exhausted")
        page = self.free.pop()
        assert self.refcount[page] == 0
        self.refcount[page] = 1
        return page

    def release(self, page: int):
        self.refcount[page] -= 1
        if self.refcount[page] == 0:
            self.free.append(page)

    # -- requests (transaction.py:50-102)
    def new(self, length: int) -> int:
        """Register a request of `length` prefix tokens; allocates its pages."""
        count = (length + PAGE_SIZE - 1) // PAGE_SIZE
        if len(self.free) < count:
            raise RuntimeError("KV page pool exhausted")
        request = self._next_request
        self._next_request += 1
        self.pages[request] = [self.alloc() for _ in range(count)]
        self.lengths[request] = length
        return request

    def fork(self, source: int) -> int:
        request = self._next_request
        self._next_request += 1
        self.pages[request] = self.pages[source].copy()
        self.lengths[request] = self.lengths[source]
        for page in self.pages[request]:
            self.refcount[page] += 1
        return request

    def checkpoint(self, request: int) -> Snapshot:
        pages = self.pages[request].copy()
        for page in pages:
            self.refcount[page] += 1
        return Snapshot(request, pages, self.lengths[request])

    def rollback(self, snapshot: Snapshot):
        if not snapshot.active:
            raise RuntimeError("snapshot already consumed")
        for page in self.pages[snapshot.request]:
            self.release(page)
        self.pages[snapshot.request] = snapshot.pages
        self.lengths[snapshot.request] = snapshot.length
        snapshot.active = False

    def accept(self, snapshot: Snapshot):
        if not snapshot.active:
            raise RuntimeError("snapshot already consumed")
        for page in snapshot.pages:
            self.release(page)
        snapshot.active = False

    # -- commit planning (transaction.py:114-150)
    def plan_commit(self, request: int, path_len: int, plan: CommitPlan,
                    draft_index: int, path: list[int]):
        """Apply one request's commit to the page state and append its device
        work to `plan`. Raises exactly where the reference raises."""
        old_length = self.lengths[request]
        old_pages = self.pages[request]
        new_page_count = (old_length + path_len + PAGE_SIZE - 1) // PAGE_SIZE
        copy_partial = old_length % PAGE_SIZE != 0 and self.refcount[old_pages[-1]] > 1
        pages_needed = new_page_count - len(old_pages) + int(copy_partial)
        if len(self.free) < pages_needed:
            raise RuntimeError("KV page pool exhausted")
        if copy_partial:
            old = old_pages[-1]
            fresh = self.alloc()
            plan.clone_src.append(old)
            plan.clone_dst.append(fresh)
            old_pages[-1] = fresh
            self.release(old)
        while len(old_pages) < new_page_count:
            old_pages.append(self.alloc())
        for i, node in enumerate(path):
            pos = old_length + i
            plan.entry_request.append(draft_index)
            plan.entry_node.append(node)
            plan.entry_page.append(old_pages[pos // PAGE_SIZE])
            plan.entry_slot.append(pos % PAGE_SIZE)
        self.lengths[request] += path_len

    def plan_commit_batch(self, commits, nodes: int) -> CommitPlan:
        """commits: iterable of (request, path, draft_index) applied in order.
        Validates like transaction.py:116-121. All or nothing: if any commit
        of the batch fails (bad path, pool exhausted) the page state is left
        exactly as it was and the error is raised."""
        saved = (self.refcount.copy(), self.free.copy(),
                 {r: p.copy() for r, p in self.pages.items()}, dict(self.lengths))
        plan = CommitPlan()
        try:
            for request, path, draft_index in commits:
                path = [int(n) for n in path]
                if not path or len(path) > nodes:
                    raise ValueError("path is empty or longer than draft")
                if any(n < 0 or n >= nodes for n in path):
                    raise ValueError("path node out of range")
                self.plan_commit(request, len(path), plan, draft_index, path)
        except Exception:
            self.refcount, self.free, self.pages, self.lengths = saved
            raise
        return plan

    def page_table(self, requests, width: int | None = None, fill: int = -1):
        rows = [self.pages[r] for r in requests]
        width = width or max(1, max(len(r) for r in rows))
        return [r + [fill] * (width - len(r)) for r in rows]
