"""Seeded synthetic workloads with the shapes of the BASELINE configurations.

No dataset is involved anywhere: every tensor is drawn from N(0, 1) (FP16)
with numpy's PCG64 generator and a fixed seed, so the CUDA path, the CPU oracle
and the reference's CPU code all see identical bytes.
"""
from __future__ import annotations

import numpy as np

from bc_cow import CommitPlan, PagePool

PAGE = 16
KV_TOKEN_BYTES = 8 * 128 * 2 * 2  # K + V of one token, Hkv=8, D=128, FP16


def rand_half(rng: np.random.Generator, shape) -> np.ndarray:
    """N(0,1) values rounded to FP16, as uint16 bit patterns."""
    return rng.standard_normal(shape, dtype=np.float32).astype(np.float16).view(np.uint16)


def random_parents(rng, nodes: int) -> np.ndarray:
    """parent[0] = -1 (root), parent[i] uniform over [0, i-1]."""
    par = np.empty(nodes, np.int32)
    par[0] = -1
    for i in range(1, nodes):
        par[i] = rng.integers(0, i)
    return par


def root_to_leaf(rng, parent: np.ndarray) -> list[int]:
    """A seeded random leaf, then its root-to-leaf path."""
    n = len(parent)
    has_child = np.zeros(n, bool)
    for i in range(1, n):
        has_child[parent[i]] = True
    leaves = np.flatnonzero(~has_child)
    cur = int(leaves[rng.integers(0, len(leaves))])
    path = []
    while cur >= 0:
        path.append(cur)
        cur = int(parent[cur])
    return path[::-1]


class TreeCowWorkload:
    """`batch` requests share one physical prefix of
    `prefix` tokens (the last page partial: 2040 = 127 pages + 8 tokens); each
    request has its own random `nodes`-node tree and a seeded accepted
    root-to-leaf path, committed copy-on-write in request order.

    The page owner follows the reference PagedTreeCache: request 0 is created
    from the prefix, requests 1.. are forks of it.
    """

    def __init__(self, seed=2040, batch=8, prefix=2040, nodes=7, hq=32, hkv=8, dim=128,
                 pool_pages=256):
        rng = np.random.default_rng(seed)
        self.batch, self.prefix, self.nodes = batch, prefix, nodes
        self.hq, self.hkv, self.dim, self.pool_pages = hq, hkv, dim, pool_pages
        self.prefix_k = rand_half(rng, (prefix, hkv, dim))
        self.prefix_v = rand_half(rng, (prefix, hkv, dim))
        self.draft_q = rand_half(rng, (batch, nodes, hq, dim))
        self.draft_k = rand_half(rng, (batch, nodes, hkv, dim))
        self.draft_v = rand_half(rng, (batch, nodes, hkv, dim))
        self.parent = np.stack([random_parents(rng, nodes) for _ in range(batch)])
        self.paths = [root_to_leaf(rng, self.parent[b]) for b in range(batch)]

        self.pool = PagePool(pool_pages)
        self.requests = [self.pool.new(prefix)]
        self.requests += [self.pool.fork(self.requests[0]) for _ in range(batch - 1)]
        self.prefix_pages = list(self.pool.pages[self.requests[0]])
        self.max_pages = (prefix + nodes + PAGE - 1) // PAGE
        self.pages = np.array(self.pool.page_table(self.requests, self.max_pages), np.int32)
        self.lengths = np.full(batch, prefix, np.int32)

    def initial_cache(self):
        """K/V pools [P, 16, Hkv, D] (uint16) holding the prefix pages."""
        k = np.zeros((self.pool_pages, PAGE, self.hkv, self.dim), np.uint16)
        v = np.zeros_like(k)
        for i, page in enumerate(self.prefix_pages):
            n = min(PAGE, self.prefix - i * PAGE)
            k[page, :n] = self.prefix_k[i * PAGE:i * PAGE + n]
            v[page, :n] = self.prefix_v[i * PAGE:i * PAGE + n]
        return k, v

    def plan(self) -> tuple[CommitPlan, PagePool]:
        """The commit plan of the whole batch, from a fresh copy of the pool."""
        pool = PagePool(self.pool_pages)
        reqs = [pool.new(self.prefix)] + [pool.fork(0) for _ in range(self.batch - 1)]
        plan = pool.plan_commit_batch(
            [(reqs[b], self.paths[b], b) for b in range(self.batch)], self.nodes)
        return plan, pool

    def shape(self):
        return (self.batch, self.hq, self.hkv, self.dim, self.max_pages, self.pool_pages)

    def verify_bytes(self) -> int:
        """Algorithmic bytes of one tree_verify launch: the shared prefix K/V
        once, draft K/V, draft Q, FP32 output, page table, lengths, parents."""
        b, n, hq, hkv, d = self.batch, self.nodes, self.hq, self.hkv, self.dim
        prefix_kv = self.prefix * hkv * d * 2 * 2
        return (prefix_kv + b * n * hkv * d * 2 * 2 + b * n * hq * d * 2 + b * n * hq * d * 4
                + b * self.max_pages * 4 + b * 4 + b * n * 4)

    def commit_bytes(self, plan: CommitPlan) -> int:
        page_bytes = PAGE * self.hkv * self.dim * 2 * 2
        row_bytes = self.hkv * self.dim * 2 * 2
        return 2 * page_bytes * len(plan.clone_src) + 2 * row_bytes * len(plan.entry_node)

    def verify_flops(self) -> int:
        depth_sum = sum(len(root_to_leaf_all(self.parent[b], i)) for b in range(self.batch)
                        for i in range(self.nodes))
        per_key = 4 * self.dim  # QK and PV multiply-adds
        return self.hq * per_key * (self.batch * self.nodes * self.prefix + depth_sum)


def root_to_leaf_all(parent, node):
    path = []
    cur = node
    while cur >= 0:
        path.append(cur)
        cur = int(parent[cur])
    return path
