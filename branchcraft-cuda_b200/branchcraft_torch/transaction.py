"""Copy-on-write page transaction for tree verification.

`PagedTreeCache` keeps the reference's API and ownership rules
(python/branchcraft_torch/transaction.py): snapshots own page references, so
committing to a shared or remembered partial page allocates a copy, and a
rollback restores both page mappings and the previous bytes. Page bookkeeping
is `bc_cow.PagePool`; every device copy goes through the branchcraft ops.

Added: `commit_batch`, which commits many requests' accepted paths with one
plan and two kernel launches instead of one torch copy plus one launch per
request.
"""
from __future__ import annotations

import torch

from bc_cow import CommitPlan, PagePool, Snapshot

from . import commit_batch_, commit_path_, tree_verify

__all__ = ["PagedTreeCache", "Snapshot"]


class PagedTreeCache:
    def __init__(self, physical_pages: int, kv_heads: int, head_dim: int, device: str = "cuda"):
        if head_dim not in (64, 128) or physical_pages < 1:
            raise ValueError("head_dim must be 64/128; physical_pages must be positive")
        self.k = torch.zeros((physical_pages, 16, kv_heads, head_dim), device=device,
                             dtype=torch.float16)
        self.v = torch.zeros_like(self.k)
        self.pool = PagePool(physical_pages)

    # The reference exposes these attributes directly.
    @property
    def refcount(self):
        return self.pool.refcount

    @property
    def free(self):
        return self.pool.free

    @property
    def pages(self):
        return self.pool.pages

    @property
    def lengths(self):
        return self.pool.lengths

    def new(self, prefix_k: torch.Tensor, prefix_v: torch.Tensor) -> int:
        """Create one request from [tokens, KV heads, head dim] FP16 tensors."""
        if prefix_k.shape != prefix_v.shape or prefix_k.ndim != 3:
            raise ValueError("prefix K/V shapes must match [tokens, heads, dim]")
        if prefix_k.dtype != torch.float16 or prefix_k.device != self.k.device:
            raise ValueError("prefix must be FP16 on the cache device")
        if tuple(prefix_k.shape[1:]) != tuple(self.k.shape[2:]):
            raise ValueError("prefix head shape differs from cache")
        n = prefix_k.shape[0]
        request = self.pool.new(n)
        for i, page in enumerate(self.pool.pages[request]):
            m = min(16, n - i * 16)
            self.k[page, :m].copy_(prefix_k[i * 16:i * 16 + m])
            self.v[page, :m].copy_(prefix_v[i * 16:i * 16 + m])
        return request

    def fork(self, source: int) -> int:
        return self.pool.fork(source)

    def checkpoint(self, request: int) -> Snapshot:
        return self.pool.checkpoint(request)

    def rollback(self, snapshot: Snapshot):
        self.pool.rollback(snapshot)

    def accept(self, snapshot: Snapshot):
        self.pool.accept(snapshot)

    def verify(self, request: int, q: torch.Tensor, draft_k: torch.Tensor,
               draft_v: torch.Tensor, parent: torch.Tensor) -> torch.Tensor:
        """Verify one request; draft inputs have leading batch dimension 1."""
        pages = self.pool.pages[request] or [0]  # ignored when prefix length is zero
        page_table = torch.tensor([pages], device=self.k.device, dtype=torch.int32)
        length = torch.tensor([self.pool.lengths[request]], device=self.k.device,
                              dtype=torch.int32)
        return tree_verify(q, self.k, self.v, page_table, length, draft_k, draft_v, parent)

    def verify_batch(self, requests, q, draft_k, draft_v, parent) -> torch.Tensor:
        """Verify several requests in one launch; draft inputs are [len(requests), N, ...].
        Requests sharing identical page tables share every K/V tile on the GPU."""
        width = max(1, max(len(self.pool.pages[r]) for r in requests))
        table = self.pool.page_table(requests, width, fill=0)
        page_table = torch.tensor(table, device=self.k.device, dtype=torch.int32)
        lengths = torch.tensor([self.pool.lengths[r] for r in requests], device=self.k.device,
                               dtype=torch.int32)
        return tree_verify(q, self.k, self.v, page_table, lengths, draft_k, draft_v, parent)

    def commit(self, request: int, path: list[int], draft_k: torch.Tensor,
               draft_v: torch.Tensor):
        """Append an accepted root-to-leaf path, preserving shared pages."""
        if not path or len(path) > draft_k.shape[1]:
            raise ValueError("path is empty or longer than draft")
        if draft_k.shape != draft_v.shape or draft_k.shape[0] != 1:
            raise ValueError("draft K/V must match and have batch size 1")
        if any(node < 0 or node >= draft_k.shape[1] for node in path):
            raise ValueError("path node out of range")
        plan = CommitPlan()
        self.pool.plan_commit(request, len(path), plan, 0, list(path))
        self._execute(plan, draft_k, draft_v, single=True)

    def commit_batch(self, commits, draft_k: torch.Tensor, draft_v: torch.Tensor) -> CommitPlan:
        """commits: [(request, path, draft_index)] applied in order; draft_k/v are
        [B, N, Hkv, D]. Same page-table result as calling commit() in order."""
        if draft_k.shape != draft_v.shape:
            raise ValueError("draft K/V must match")
        plan = self.pool.plan_commit_batch(commits, draft_k.shape[1])
        self._execute(plan, draft_k, draft_v, single=False)
        return plan

    def _execute(self, plan: CommitPlan, draft_k, draft_v, single: bool):
        dev = self.k.device

        def t(xs):
            return torch.tensor(xs, device=dev, dtype=torch.int32)

        if single and not plan.clone_src:
            commit_path_(self.k, self.v, draft_k, draft_v, t(plan.entry_node),
                         t(plan.entry_page), t(plan.entry_slot), 0)
            return
        commit_batch_(self.k, self.v, draft_k, draft_v, t(plan.clone_src), t(plan.clone_dst),
                      t(plan.entry_request), t(plan.entry_node), t(plan.entry_page),
                      t(plan.entry_slot))
