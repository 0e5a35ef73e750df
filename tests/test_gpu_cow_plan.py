"""The device copy-on-write planner (bc_cow_plan) against the host planner
(bc_cow.PagePool.plan_commit_batch, itself pinned to the sequential oracle of
the reference's PagedTreeCache in test_cow_planner.py): on random transaction
histories the device produces the same clones, entries, page tables, lengths,
refcounts and free list, bit for bit; failed batches (a bad path, too few
free pages) leave the device state unchanged, as the reference's errors leave
its pool; and bc_tree_step runs a whole config-2 step (plan, verification and
commit) from device state with the sequential result."""
import numpy as np
import pytest
import torch

import bc_testutil as U
import oracle as O
from bc_cow import PagePool
from cow_oracle import CowOracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def capi():
    import bc_capi

    return bc_capi


def _i32(x):
    return torch.tensor(np.asarray(x, np.int32), device="cuda")


def _device_state(pool: PagePool):
    return (_i32(pool.refcount), _i32(pool.free + [0] * (pool.physical_pages - len(pool.free))),
            _i32([len(pool.free)]))


def _batch_inputs(pool, reqs, paths, nodes, width):
    pages = _i32(pool.page_table(reqs, width))
    lengths = _i32([pool.lengths[r] for r in reqs])
    plen = _i32([len(p) for p in paths])
    pn = np.full((len(reqs), nodes), -1, np.int32)
    for b, p in enumerate(paths):  # (a path longer than `nodes` is cut; its length stays)
        pn[b, :min(len(p), nodes)] = p[:nodes]
    return pages, lengths, plen, _i32(pn)


def _run_device(capi, pool, reqs, paths, nodes, width_in, width_out):
    rc, stack, nfree = _device_state(pool)
    pages, lengths, plen, pn = _batch_inputs(pool, reqs, paths, nodes, width_in)
    plan = capi.CowPlan(len(reqs), nodes, width_out)
    capi.cow_plan(pages, lengths, plen, pn, (rc, stack, nfree), plan, pool.physical_pages)
    torch.cuda.synchronize()
    return plan, rc, stack, nfree


def _assert_matches(pool, plan_host, reqs, plan, rc, stack, nfree, width_out):
    cnt = plan.counts.cpu().tolist()
    assert cnt[2] == 0
    ncl, nent = cnt[0], cnt[1]
    assert plan.clone_src[:ncl].tolist() == plan_host.clone_src
    assert plan.clone_dst[:ncl].tolist() == plan_host.clone_dst
    assert plan.entry_request[:nent].tolist() == plan_host.entry_request
    assert plan.entry_node[:nent].tolist() == plan_host.entry_node
    assert plan.entry_page[:nent].tolist() == plan_host.entry_page
    assert plan.entry_slot[:nent].tolist() == plan_host.entry_slot
    assert plan.pages_out.tolist() == pool.page_table(reqs, width_out)
    assert plan.lengths_out.tolist() == [pool.lengths[r] for r in reqs]
    assert rc.tolist() == pool.refcount
    n = int(nfree.item())
    assert stack[:n].tolist() == pool.free


@pytest.mark.parametrize("seed", range(12))
def test_random_histories_match_host_planner(capi, seed):
    """Random new / fork / checkpoint / rollback / accept histories; every
    batch commit planned on the device from the host's state, then on the
    host, and compared."""
    rng = np.random.default_rng(seed)
    P, N = 64, 7
    pool = PagePool(P)
    live, snaps, batches = [], [], 0
    for _ in range(60):
        op = rng.choice(["new", "fork", "snap", "batch", "batch", "rollback", "accept"])
        if op == "new" or not live:
            try:
                live.append(pool.new(int(rng.integers(1, 40))))
            except RuntimeError:
                pass
        elif op == "fork":
            live.append(pool.fork(int(rng.choice(live))))
        elif op == "snap":
            snaps.append(pool.checkpoint(int(rng.choice(live))))
        elif op == "batch":
            reqs = [int(x) for x in rng.choice(live, size=min(len(live), 4), replace=False)]
            paths = [list(int(n) for n in rng.choice(N, size=int(rng.integers(1, N + 1)),
                                                       replace=False)) for _ in reqs]
            width_in = max(1, max(len(pool.pages[r]) for r in reqs))
            width_out = width_in + 2
            plan, rc, stack, nfree = _run_device(capi, pool, reqs, paths, N, width_in, width_out)
            before = (pool.refcount.copy(), pool.free.copy())
            try:
                host = pool.plan_commit_batch([(r, paths[i], i) for i, r in enumerate(reqs)], N)
            except RuntimeError:
                assert plan.counts[2].item() == 2  # exhausted, state unchanged
                assert rc.tolist() == before[0]
                assert stack[:int(nfree.item())].tolist() == before[1]
                continue
            _assert_matches(pool, host, reqs, plan, rc, stack, nfree, width_out)
            batches += 1
        elif op == "rollback" and snaps:
            pool.rollback(snaps.pop(int(rng.integers(len(snaps)))))
        elif op == "accept" and snaps:
            pool.accept(snaps.pop(int(rng.integers(len(snaps)))))
    assert batches > 0


def test_bad_paths_change_nothing(capi):
    pool = PagePool(8)
    a = pool.new(20)
    b = pool.fork(a)
    for paths in ([[0], []], [[0, 9], [1]], [[0] * 8, [1]]):
        plan, rc, stack, nfree = _run_device(capi, pool, [a, b], paths, 7, 2, 4)
        assert plan.counts.tolist()[:3] == [0, 0, 1]
        assert rc.tolist() == pool.refcount
        assert stack[:int(nfree.item())].tolist() == pool.free


def test_exhausted_pool_changes_nothing(capi):
    pool = PagePool(5)
    a = pool.new(20)            # pages 0, 1 (the second partial)
    pool.fork(a)
    c = pool.new(40)            # pages 2, 3, 4: nothing left
    plan, rc, stack, nfree = _run_device(capi, pool, [c, a], [[0], [0]], 7, 3, 4)
    assert plan.counts.tolist()[:3] == [0, 0, 2]  # a's clone needs a free page
    assert rc.tolist() == pool.refcount and int(nfree.item()) == 0


def test_config2_step_from_device_state(capi):
    """BASELINE config 2 in one call: the device plans the 8 commits from the
    pool state (7 clones, the 8th in place), verifies and commits; the
    verification equals the unfused verify, the cache the sequential oracle's,
    the new page tables and state the host planner's."""
    from bc_workloads import TreeCowWorkload

    wl = TreeCowWorkload(seed=2040)
    pool = PagePool(wl.pool_pages)
    reqs = [pool.new(wl.prefix)] + [pool.fork(0) for _ in range(wl.batch - 1)]
    rc, stack, nfree = _device_state(pool)
    k0, v0 = wl.initial_cache()
    ck, cv = U.to_dev(k0), U.to_dev(v0)
    s = capi.make_shape(*wl.shape())
    t = {n: U.to_dev(getattr(wl, n)) for n in ("draft_q", "draft_k", "draft_v", "parent",
                                               "pages", "lengths")}
    plen = _i32([len(p) for p in wl.paths])
    pn = np.full((wl.batch, wl.nodes), -1, np.int32)
    for b, p in enumerate(wl.paths):
        pn[b, :len(p)] = p
    plan = capi.CowPlan(wl.batch, wl.nodes, wl.max_pages)
    out = torch.full((wl.batch, wl.nodes, wl.hq, wl.dim), float("nan"), device="cuda")
    capi.last_device_error()
    capi.tree_step(s, t["draft_q"], ck, cv, t["pages"], t["lengths"], t["draft_k"], t["draft_v"],
                   t["parent"], out, wl.nodes, plen, _i32(pn), (rc, stack, nfree), plan)
    torch.cuda.synchronize()
    assert capi.last_device_error() == 0
    assert plan.counts.tolist()[:3] == [7, sum(len(p) for p in wl.paths), 0]
    ref = torch.empty_like(out)
    capi.tree_verify(s, t["draft_q"], U.to_dev(k0), U.to_dev(v0), t["pages"], t["lengths"],
                     t["draft_k"], t["draft_v"], t["parent"], ref, wl.nodes)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    expected = O.tree(wl.shape(), wl.nodes, wl.draft_q, k0, v0, wl.pages, wl.lengths,
                      wl.draft_k, wl.draft_v, wl.parent)
    U.assert_close_baseline(out.cpu().numpy(), expected)
    host = pool.plan_commit_batch([(reqs[b], wl.paths[b], b) for b in range(wl.batch)], wl.nodes)
    _assert_matches(pool, host, reqs, plan, rc, stack, nfree, wl.max_pages)
    cow = CowOracle(wl.pool_pages, wl.hkv, wl.dim)
    r0 = cow.new(wl.prefix_k, wl.prefix_v)
    oreqs = [r0] + [cow.fork(r0) for _ in range(wl.batch - 1)]
    for b in range(wl.batch):
        cow.commit(oreqs[b], wl.paths[b], wl.draft_k[b], wl.draft_v[b])
    assert np.array_equal(U.half_bits(ck), cow.k)
    assert np.array_equal(U.half_bits(cv), cow.v)
    assert plan.pages_out.tolist() == [cow.pages[r] + [-1] * (wl.max_pages - len(cow.pages[r]))
                                       for r in oreqs]


def test_state_out_keeps_the_state_in(capi):
    """With separate output arrays the input state is left as it was (and a
    failed batch writes the input state to the outputs)."""
    pool = PagePool(16)
    a = pool.new(20)
    b = pool.fork(a)
    rc, stack, nfree = _device_state(pool)
    rc2, stack2, nfree2 = (torch.full_like(x, -7) for x in (rc, stack, nfree))
    pages, lengths, plen, pn = _batch_inputs(pool, [a, b], [[0, 1], [2]], 7, 2)
    plan = capi.CowPlan(2, 7, 4)
    capi.cow_plan(pages, lengths, plen, pn, (rc, stack, nfree), plan, 16,
                  state_out=(rc2, stack2, nfree2))
    torch.cuda.synchronize()
    host = pool.plan_commit_batch([(a, [0, 1], 0), (b, [2], 1)], 7)
    assert plan.counts.tolist()[:3] == [1, 3, 0] and plan.clone_dst[:1].tolist() == host.clone_dst
    assert rc.tolist() != pool.refcount  # the input state is untouched
    assert rc2.tolist() == pool.refcount and stack2[:int(nfree2.item())].tolist() == pool.free
    # a failed batch: the outputs receive the input state
    rc3, stack3, nfree3 = (torch.full_like(x, -7) for x in (rc, stack, nfree))
    pages, lengths, plen, pn = _batch_inputs(pool, [a], [[]], 7, 2)
    capi.cow_plan(pages, lengths, plen, pn, (rc2, stack2, nfree2), plan, 16,
                  state_out=(rc3, stack3, nfree3))
    torch.cuda.synchronize()
    assert plan.counts.tolist()[:3] == [0, 0, 1]
    assert rc3.tolist() == rc2.tolist() and nfree3.tolist() == nfree2.tolist()


@pytest.mark.parametrize("batch,prefix,pool_pages", [
    (80, 300, 2048),   # 160 CTAs: more than one wave, so the planner is its own launch
    (6, 40, 64),       # one wave: planned inside the verify launch
])
def test_tree_step_both_planner_placements(capi, batch, prefix, pool_pages):
    """bc_tree_step where the plan is made inside the verify launch (a one-wave
    grid) and where it cannot be (a grid of several waves): the same
    sequential result either way — plan, state and tables equal the host
    planner's, the cache the oracle's, the output the unfused verify's."""
    rng = np.random.default_rng(batch + prefix)
    hq, hkv, dim, nodes = 32, 8, 128, 7
    pool = PagePool(pool_pages)
    reqs = []
    for b in range(batch):  # pairs sharing a prefix, lengths not page-aligned
        reqs.append(pool.new(prefix + 3 * (b // 2)) if b % 2 == 0 else pool.fork(reqs[-1]))
    width = max(len(pool.pages[r]) for r in reqs)
    width_out = width + 2
    ora = CowOracle(pool_pages, hkv, dim)
    k0 = U.rand_half(rng, (pool_pages, 16, hkv, dim))
    v0 = U.rand_half(rng, (pool_pages, 16, hkv, dim))
    ora.k[:], ora.v[:] = k0, v0
    parent = U.random_tree_parents(rng, batch, nodes)
    paths = []
    for b in range(batch):
        cur, path = int(rng.integers(0, nodes)), []
        while cur >= 0:
            path.append(cur)
            cur = int(parent[b, cur])
        paths.append(path[::-1])
    draft_q = U.rand_half(rng, (batch, nodes, hq, dim))
    draft_k = U.rand_half(rng, (batch, nodes, hkv, dim))
    draft_v = U.rand_half(rng, (batch, nodes, hkv, dim))
    rc, stack, nfree = _device_state(pool)
    pages, lengths, plen, pn = _batch_inputs(pool, reqs, paths, nodes, width)
    s = capi.make_shape(batch, hq, hkv, dim, width, pool_pages)
    t = {"draft_q": U.to_dev(draft_q), "draft_k": U.to_dev(draft_k), "draft_v": U.to_dev(draft_v),
         "parent": U.to_dev(parent)}
    ck, cv = U.to_dev(k0), U.to_dev(v0)
    plan = capi.CowPlan(batch, nodes, width_out)
    out = torch.full((batch, nodes, hq, dim), float("nan"), device="cuda")
    capi.last_device_error()
    capi.tree_step(s, t["draft_q"], ck, cv, pages, lengths, t["draft_k"], t["draft_v"],
                   t["parent"], out, nodes, plen, pn, (rc, stack, nfree), plan)
    ref = torch.empty_like(out)
    capi.tree_verify(s, t["draft_q"], U.to_dev(k0), U.to_dev(v0), pages, lengths, t["draft_k"],
                     t["draft_v"], t["parent"], ref, nodes)
    torch.cuda.synchronize()
    assert capi.last_device_error() == 0
    assert torch.equal(out, ref)
    host = pool.plan_commit_batch([(reqs[b], paths[b], b) for b in range(batch)], nodes)
    _assert_matches(pool, host, reqs, plan, rc, stack, nfree, width_out)
    # the oracle executes the host plan on the same bytes
    for src, dst in zip(host.clone_src, host.clone_dst):
        ora.k[dst], ora.v[dst] = ora.k[src], ora.v[src]
    for r, n, pg, sl in zip(host.entry_request, host.entry_node, host.entry_page, host.entry_slot):
        ora.k[pg, sl], ora.v[pg, sl] = draft_k[r, n], draft_v[r, n]
    assert np.array_equal(U.half_bits(ck), ora.k)
    assert np.array_equal(U.half_bits(cv), ora.v)


def test_tree_step_graph_replays_with_new_paths(capi):
    """bc_tree_step captured once in a CUDA graph and replayed with other
    accepted paths written into the same buffers before each replay (the pool
    state and cache restored): every replay plans its own paths. The plan
    flag inside the launch must start each replay unpublished (counts[3] and
    counts[4] are back at zero after every launch), or a replay's commit
    would read the plan of the replay before."""
    import copy

    rng = np.random.default_rng(77)
    batch, prefix, pool_pages = 6, 40, 64
    hq, hkv, dim, nodes = 32, 8, 128, 7
    pool = PagePool(pool_pages)
    reqs = []
    for b in range(batch):
        reqs.append(pool.new(prefix + 3 * (b // 2)) if b % 2 == 0 else pool.fork(reqs[-1]))
    width = max(len(pool.pages[r]) for r in reqs)
    width_out = width + 2
    k0 = U.rand_half(rng, (pool_pages, 16, hkv, dim))
    v0 = U.rand_half(rng, (pool_pages, 16, hkv, dim))
    parent = U.random_tree_parents(rng, batch, nodes)

    def random_paths():
        paths = []
        for b in range(batch):
            cur, path = int(rng.integers(0, nodes)), []
            while cur >= 0:
                path.append(cur)
                cur = int(parent[b, cur])
            paths.append(path[::-1])
        return paths

    draft_q = U.rand_half(rng, (batch, nodes, hq, dim))
    draft_k = U.rand_half(rng, (batch, nodes, hkv, dim))
    draft_v = U.rand_half(rng, (batch, nodes, hkv, dim))
    state_in = _device_state(pool)
    state_out = tuple(torch.zeros_like(x) for x in state_in)
    pages, lengths, plen, pn = _batch_inputs(pool, reqs, random_paths(), nodes, width)
    s = capi.make_shape(batch, hq, hkv, dim, width, pool_pages)
    t = {"draft_q": U.to_dev(draft_q), "draft_k": U.to_dev(draft_k), "draft_v": U.to_dev(draft_v),
         "parent": U.to_dev(parent)}
    k0d, v0d = U.to_dev(k0), U.to_dev(v0)
    ck, cv = k0d.clone(), v0d.clone()
    plan = capi.CowPlan(batch, nodes, width_out)
    out = torch.empty((batch, nodes, hq, dim), device="cuda")
    capi.last_device_error(reset=True)
    step = lambda: capi.tree_step(s, t["draft_q"], ck, cv, pages, lengths, t["draft_k"],
                                  t["draft_v"], t["parent"], out, nodes, plen, pn, state_in,
                                  plan, state_out=state_out)
    step()  # warm the library's per-device caches outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(6):
        paths = random_paths()
        _, _, plen_h, pn_h = _batch_inputs(pool, reqs, paths, nodes, width)
        plen.copy_(plen_h)
        pn.copy_(pn_h)
        ck.copy_(k0d)
        cv.copy_(v0d)
        for x in state_out:
            x.fill_(-1)
        g.replay()
        torch.cuda.synchronize()
        assert capi.last_device_error() == 0
        assert plan.counts[3:].tolist() == [0, 0]
        expect = copy.deepcopy(pool)
        host = expect.plan_commit_batch([(reqs[b], paths[b], b) for b in range(batch)], nodes)
        _assert_matches(expect, host, reqs, plan, *state_out, width_out)
        ka, va = k0.copy(), v0.copy()
        for src, dst in zip(host.clone_src, host.clone_dst):
            ka[dst], va[dst] = ka[src], va[src]
        for r, n, pg, sl in zip(host.entry_request, host.entry_node, host.entry_page,
                                host.entry_slot):
            ka[pg, sl], va[pg, sl] = draft_k[r, n], draft_v[r, n]
        assert np.array_equal(U.half_bits(ck), ka)
        assert np.array_equal(U.half_bits(cv), va)


def test_tree_step_serving_loop_on_device_state(capi):
    """Eight speculative steps of a 6-request batch (pairs sharing prefixes)
    driven by device state alone: every step's bc_tree_step reads the page
    tables and the pool state the step before wrote (the state updated in
    place, the tables from the previous plan's output) and commits into the
    same cache. After every step the tables and the state equal the host
    planner's, the output the oracle's verification of the cache as it was
    before the step, and the cache the bytes of the sequential commits."""
    rng = np.random.default_rng(123)
    B, hq, hkv, dim, N, P, W = 6, 8, 2, 64, 7, 160, 24
    pool = PagePool(P)
    reqs = []
    for b in range(B):
        reqs.append(pool.new(30 + 7 * b) if b % 2 == 0 else pool.fork(reqs[-1]))
    k_ref = U.rand_half(rng, (P, 16, hkv, dim))
    v_ref = U.rand_half(rng, (P, 16, hkv, dim))
    ck, cv = U.to_dev(k_ref), U.to_dev(v_ref)
    state = _device_state(pool)
    pages_h = np.array(pool.page_table(reqs, W), np.int32)
    lens_h = np.array([pool.lengths[r] for r in reqs], np.int32)
    pages, lengths = _i32(pages_h), _i32(lens_h)
    s = capi.make_shape(B, hq, hkv, dim, W, P)
    plans = [capi.CowPlan(B, N, W), capi.CowPlan(B, N, W)]
    capi.last_device_error(reset=True)
    for step in range(8):
        plan = plans[step % 2]  # (the other holds this step's input tables)
        parent = U.random_tree_parents(rng, B, N)
        paths = []
        for b in range(B):
            cur, path = int(rng.integers(0, N)), []
            while cur >= 0:
                path.append(cur)
                cur = int(parent[b, cur])
            paths.append(path[::-1])
        dq = U.rand_half(rng, (B, N, hq, dim))
        dk = U.rand_half(rng, (B, N, hkv, dim))
        dv = U.rand_half(rng, (B, N, hkv, dim))
        _, _, plen, pn = _batch_inputs(pool, reqs, paths, N, W)
        expected = O.tree((B, hq, hkv, dim, W, P), N, dq, k_ref, v_ref, pages_h, lens_h,
                          dk, dv, parent)
        out = torch.empty((B, N, hq, dim), device="cuda")
        capi.tree_step(s, U.to_dev(dq), ck, cv, pages, lengths, U.to_dev(dk), U.to_dev(dv),
                       U.to_dev(parent), out, N, plen, pn, state, plan)
        torch.cuda.synchronize()
        assert capi.last_device_error() == 0, step
        host = pool.plan_commit_batch([(reqs[b], paths[b], b) for b in range(B)], N)
        _assert_matches(pool, host, reqs, plan, *state, W)
        assert U.max_abs(out.cpu().numpy(), expected) < 2e-4, step
        for src, dst in zip(host.clone_src, host.clone_dst):
            k_ref[dst], v_ref[dst] = k_ref[src], v_ref[src]
        for r, n, pg, sl in zip(host.entry_request, host.entry_node, host.entry_page,
                                host.entry_slot):
            k_ref[pg, sl], v_ref[pg, sl] = dk[r, n], dv[r, n]
        assert np.array_equal(U.half_bits(ck), k_ref), step
        assert np.array_equal(U.half_bits(cv), v_ref), step
        # the next step reads the tables this one wrote
        pages, lengths = plan.pages_out, plan.lengths_out
        pages_h, lens_h = pages.cpu().numpy(), lengths.cpu().numpy()


def test_planner_at_its_maximum_sizes(capi):
    """bc_cow_plan at batch 256 and 256-node paths (the planner's limits):
    128 shared-prefix pairs with ragged lengths, every request committing a
    path of up to 256 nodes — the same plan, tables and state as the host
    planner, bit for bit."""
    rng = np.random.default_rng(256)
    B, N = 256, 256
    P = 8192
    pool = PagePool(P)
    reqs = []
    for b in range(B):
        reqs.append(pool.new(int(rng.integers(1, 300))) if b % 2 == 0 else pool.fork(reqs[-1]))
    paths = []
    for b in range(B):
        L = int(rng.integers(1, N + 1))
        paths.append([int(x) for x in rng.choice(N, size=L, replace=False)])
    width_in = max(len(pool.pages[r]) for r in reqs)
    width_out = width_in + (N + 15) // 16 + 1
    plan, rc, stack, nfree = _run_device(capi, pool, reqs, paths, N, width_in, width_out)
    host = pool.plan_commit_batch([(reqs[b], paths[b], b) for b in range(B)], N)
    _assert_matches(pool, host, reqs, plan, rc, stack, nfree, width_out)
    assert plan.counts.tolist()[:3] == [len(host.clone_src), len(host.entry_node), 0]
