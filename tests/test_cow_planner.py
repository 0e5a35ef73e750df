"""The host page owner (bc_cow.PagePool) against the sequential oracle of the
reference transaction (oracle/cow_oracle.py), without a GPU: random
sequences of new / fork / checkpoint / commit / rollback / accept give the
same page tables, lengths, refcounts and free lists, and executing a batched
plan (every clone, then every write) on numpy pools reproduces the oracle's
page bytes exactly."""
import numpy as np
import pytest

from bc_cow import CommitPlan, PagePool
from cow_oracle import CowOracle


def apply_plan(k, v, plan: CommitPlan, draft_k, draft_v):
    for s, d in zip(plan.clone_src, plan.clone_dst):
        k[d] = k[s]
        v[d] = v[s]
    for r, n, p, sl in zip(plan.entry_request, plan.entry_node, plan.entry_page,
                           plan.entry_slot):
        k[p, sl] = draft_k[r, n]
        v[p, sl] = draft_v[r, n]


def random_trial(seed):
    rng = np.random.default_rng(seed)
    P, hkv, d, N = 48, 2, 8, 7
    pool = PagePool(P)
    ora = CowOracle(P, hkv, d)
    k = np.zeros((P, 16, hkv, d), np.uint16)
    v = np.zeros_like(k)
    live, snaps = [], []
    for step in range(40):
        op = rng.choice(["new", "fork", "snap", "commit", "batch", "rollback", "accept"])
        if op == "new" or not live:
            n = int(rng.integers(1, 40))
            pk = rng.integers(0, 1 << 16, (n, hkv, d), dtype=np.uint16)
            pv = rng.integers(0, 1 << 16, (n, hkv, d), dtype=np.uint16)
            try:
                r = pool.new(n)
            except RuntimeError:
                with pytest.raises(RuntimeError):
                    ora.new(pk, pv)
                continue
            r2 = ora.new(pk, pv)
            assert r == r2
            for i, page in enumerate(pool.pages[r]):
                m = min(16, n - 16 * i)
                k[page, :m] = pk[16 * i:16 * i + m]
                v[page, :m] = pv[16 * i:16 * i + m]
            live.append(r)
        elif op == "fork":
            src = int(rng.choice(live))
            assert pool.fork(src) == ora.fork(src)
            live.append(pool._next_request - 1)
        elif op == "snap":
            r = int(rng.choice(live))
            snaps.append((pool.checkpoint(r), ora.checkpoint(r)))
        elif op in ("commit", "batch"):
            reqs = [int(x) for x in rng.choice(live, size=min(len(live), 3), replace=False)]
            dk = rng.integers(0, 1 << 16, (len(reqs), N, hkv, d), dtype=np.uint16)
            dv = rng.integers(0, 1 << 16, (len(reqs), N, hkv, d), dtype=np.uint16)
            paths = [list(rng.choice(N, size=int(rng.integers(1, N + 1)), replace=False))
                     for _ in reqs]
            commits = [(r, paths[i], i) for i, r in enumerate(reqs)]
            try:
                plan = pool.plan_commit_batch(commits, N)
            except RuntimeError:
                # all-or-nothing: the pool is untouched; the oracle (one
                # request at a time) is not comparable past this point
                return
            apply_plan(k, v, plan, dk, dv)
            for i, r in enumerate(reqs):
                ora.commit(r, paths[i], dk[i], dv[i])
        elif op == "rollback" and snaps:
            a, b = snaps.pop(int(rng.integers(len(snaps))))
            pool.rollback(a)
            ora.rollback(b)
        elif op == "accept" and snaps:
            a, b = snaps.pop(int(rng.integers(len(snaps))))
            pool.accept(a)
            ora.accept(b)
        assert pool.pages == ora.pages
        assert pool.lengths == ora.lengths
        assert pool.refcount == ora.refcount
        assert pool.free == ora.free
        assert np.array_equal(k, ora.k) and np.array_equal(v, ora.v)


@pytest.mark.parametrize("seed", range(25))
def test_random_transactions_match_oracle(seed):
    random_trial(seed)


def test_config2_plan_shape():
    """8 forks of a 2040-token prefix; the first 7 commits
    clone the shared half page (ids 128..134, lowest first), the 8th writes in
    place; nothing is appended (2040 + 7 < 2048)."""
    from bc_workloads import TreeCowWorkload

    wl = TreeCowWorkload(seed=2040)
    plan, pool = wl.plan()
    assert plan.clone_src == [127] * 7
    assert plan.clone_dst == list(range(128, 135))
    assert all(pool.pages[r][-1] == 128 + r for r in range(7))
    assert pool.pages[7][-1] == 127 and pool.refcount[127] == 1
    assert [pool.lengths[r] for r in range(8)] == [2040 + len(p) for p in wl.paths]


def test_batch_is_all_or_nothing():
    pool = PagePool(5)
    a = pool.new(20)            # pages 0, 1 (second page partial)
    b = pool.fork(a)
    c = pool.new(40)            # pages 2, 3, 4: pool now empty
    before = (pool.refcount.copy(), pool.free.copy(), {r: p.copy() for r, p in pool.pages.items()},
              dict(pool.lengths))
    with pytest.raises(RuntimeError):   # a's clone needs a free page
        pool.plan_commit_batch([(c, [0], 0), (a, [0], 1)], 7)
    assert (pool.refcount, pool.free, pool.pages, pool.lengths) == before
    assert b in pool.pages


def test_errors_match_reference():
    pool = PagePool(2)
    r = pool.new(20)
    with pytest.raises(ValueError):
        pool.plan_commit_batch([(r, [], 0)], 7)
    with pytest.raises(ValueError):
        pool.plan_commit_batch([(r, [9], 0)], 7)
    with pytest.raises(RuntimeError):
        pool.new(40)
