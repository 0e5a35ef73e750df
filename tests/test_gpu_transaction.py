"""The copy-on-write transaction on the GPU: the reference's scenario
(tests/test_transaction.py) restated, and a batched commit of the BASELINE
config-2 workload checked bit-exact (page contents, page tables, lengths)
against the sequential oracle."""
import numpy as np
import pytest
import torch

import bc_testutil as U
from cow_oracle import CowOracle

pytestmark = pytest.mark.gpu


def test_shared_partial_page_commit_then_rollback():
    from branchcraft_torch.transaction import PagedTreeCache

    torch.manual_seed(17)
    store = PagedTreeCache(8, 2, 64)
    prefix_k = torch.randn(19, 2, 64, device="cuda", dtype=torch.float16)
    prefix_v = torch.randn_like(prefix_k)
    original = store.new(prefix_k, prefix_v)
    sibling = store.fork(original)
    snapshot = store.checkpoint(original)
    initial_pages = store.pages[original].copy()
    old_bytes = store.k[initial_pages[-1]].clone()
    draft_k = torch.randn(1, 7, 2, 64, device="cuda", dtype=torch.float16)
    draft_v = torch.randn_like(draft_k)
    store.commit(original, [0, 2, 6], draft_k, draft_v)
    assert store.pages[original][-1] != store.pages[sibling][-1]
    assert store.lengths[original] == 22
    torch.testing.assert_close(store.k[store.pages[original][-1], 3], draft_k[0, 0])
    torch.testing.assert_close(store.k[store.pages[original][-1], 5], draft_k[0, 6])
    torch.testing.assert_close(store.k[store.pages[sibling][-1]], old_bytes)
    store.rollback(snapshot)
    assert store.pages[original] == initial_pages
    assert store.lengths[original] == 19
    torch.testing.assert_close(store.k[store.pages[original][-1]], old_bytes)


def test_config2_batch_commit_bit_exact():
    from bc_workloads import TreeCowWorkload
    from branchcraft_torch.transaction import PagedTreeCache

    wl = TreeCowWorkload(seed=2040)
    store = PagedTreeCache(wl.pool_pages, wl.hkv, wl.dim)
    r0 = store.new(U.to_dev(wl.prefix_k), U.to_dev(wl.prefix_v))
    reqs = [r0] + [store.fork(r0) for _ in range(wl.batch - 1)]
    draft_k, draft_v = U.to_dev(wl.draft_k), U.to_dev(wl.draft_v)
    # verify the whole batch first (shared prefix), then commit every path
    out = store.verify_batch(reqs, U.to_dev(wl.draft_q), draft_k, draft_v, U.to_dev(wl.parent))
    plan = store.commit_batch([(reqs[b], wl.paths[b], b) for b in range(wl.batch)], draft_k,
                              draft_v)
    torch.cuda.synchronize()
    assert len(plan.clone_src) == wl.batch - 1  # the 8th committer writes in place

    cow = CowOracle(wl.pool_pages, wl.hkv, wl.dim)
    o0 = cow.new(wl.prefix_k, wl.prefix_v)
    oreqs = [o0] + [cow.fork(o0) for _ in range(wl.batch - 1)]
    for b in range(wl.batch):
        cow.commit(oreqs[b], wl.paths[b], wl.draft_k[b], wl.draft_v[b])
    assert [store.pages[r] for r in reqs] == [cow.pages[r] for r in oreqs]
    assert [store.lengths[r] for r in reqs] == [cow.lengths[r] for r in oreqs]
    assert store.refcount == cow.refcount and store.free == cow.free
    assert np.array_equal(U.half_bits(store.k), cow.k)
    assert np.array_equal(U.half_bits(store.v), cow.v)
    # the verify output of the batch matches the tree oracle
    import oracle as O

    k0, v0 = wl.initial_cache()
    expected = O.tree(wl.shape(), wl.nodes, wl.draft_q, k0, v0, wl.pages, wl.lengths,
                      wl.draft_k, wl.draft_v, wl.parent)
    U.assert_close_baseline(out.cpu().numpy(), expected)
