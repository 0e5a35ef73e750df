"""bc_tree_verify_commit: tree verification and the batch copy-on-write commit
in one launch. The verification must equal bc_tree_verify's bit for bit (the
commit touches no byte a verified row depends on) and the oracle at the
BASELINE tolerance; the cache after the call must equal the sequential
PagedTreeCache semantics (the reference's python/branchcraft_torch/
transaction.py:114-150, restated by oracle/cow_oracle.py) bit for bit."""
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


def _arr(x):
    return U.to_dev(np.array(x, np.int32)) if len(x) else None


def _fused(capi, shape, t, ck, cv, plan, nodes, out):
    capi.tree_verify_commit(shape, t["draft_q"], ck, cv, t["pages"], t["lengths"], t["draft_k"],
                            t["draft_v"], t["parent"], out, nodes, _arr(plan.clone_src),
                            _arr(plan.clone_dst), _arr(plan.entry_request),
                            _arr(plan.entry_node), _arr(plan.entry_page), _arr(plan.entry_slot))


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_config2_step_in_one_launch(capi, out_dtype):
    """8 requests sharing a 2040-token prefix, 7 clones of
    the shared partial page and 23 row commits, fused into the verify launch;
    then 200 more launches back to back stay clean and identical."""
    from bc_workloads import TreeCowWorkload

    wl = TreeCowWorkload(seed=2040)
    plan, _ = wl.plan()
    k0, v0 = wl.initial_cache()
    s = capi.make_shape(*wl.shape())
    t = {n: U.to_dev(getattr(wl, n)) for n in ("draft_q", "draft_k", "draft_v", "parent",
                                               "pages", "lengths")}
    # the unfused verify on the pre-commit cache
    ref_out = torch.full((wl.batch, wl.nodes, wl.hq, wl.dim), float("nan"), device="cuda",
                         dtype=out_dtype)
    capi.tree_verify(s, t["draft_q"], U.to_dev(k0), U.to_dev(v0), t["pages"], t["lengths"],
                     t["draft_k"], t["draft_v"], t["parent"], ref_out, wl.nodes)
    ck, cv = U.to_dev(k0), U.to_dev(v0)
    out = torch.full_like(ref_out, float("nan"))
    capi.last_device_error()
    _fused(capi, s, t, ck, cv, plan, wl.nodes, out)
    torch.cuda.synchronize()
    assert capi.last_device_error() == 0
    assert torch.equal(out, ref_out)
    expected = O.tree(wl.shape(), wl.nodes, wl.draft_q, k0, v0, wl.pages, wl.lengths,
                      wl.draft_k, wl.draft_v, wl.parent)
    U.assert_close_baseline(out.float().cpu().numpy(), expected)
    cow = CowOracle(wl.pool_pages, wl.hkv, wl.dim)
    r0 = cow.new(wl.prefix_k, wl.prefix_v)
    reqs = [r0] + [cow.fork(r0) for _ in range(wl.batch - 1)]
    for b in range(wl.batch):
        cow.commit(reqs[b], wl.paths[b], wl.draft_k[b], wl.draft_v[b])
    assert np.array_equal(U.half_bits(ck), cow.k)
    assert np.array_equal(U.half_bits(cv), cow.v)
    # The same step replayed 200 times: the verified rows read no byte the
    # commit writes, so the output stays identical; the cache evolves exactly
    # as under the same 201 steps run unfused (verify, then bc_commit_batch).
    # (A replayed commit is not the first one: its clones copy a source page
    # whose in-place slots the previous replay wrote.)
    for _ in range(200):
        _fused(capi, s, t, ck, cv, plan, wl.nodes, out)
    uk, uv = U.to_dev(k0), U.to_dev(v0)
    out2 = torch.empty_like(out)
    for _ in range(201):
        capi.tree_verify(s, t["draft_q"], uk, uv, t["pages"], t["lengths"], t["draft_k"],
                         t["draft_v"], t["parent"], out2, wl.nodes)
        capi.commit_batch(s, wl.nodes, t["draft_k"], t["draft_v"], uk, uv, _arr(plan.clone_src),
                          _arr(plan.clone_dst), _arr(plan.entry_request), _arr(plan.entry_node),
                          _arr(plan.entry_page), _arr(plan.entry_slot))
    torch.cuda.synchronize()
    assert capi.last_device_error() == 0
    assert torch.equal(out, ref_out) and torch.equal(out2, ref_out)
    assert torch.equal(ck, uk) and torch.equal(cv, uv)


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_random_batches_with_appends(capi, seed):
    """Small pools, D=64, random shared and private prefixes, paths that cross
    page boundaries (fresh pages appended) and clones: fused equals the
    unfused verify and the sequential copy-on-write commit."""
    rng = np.random.default_rng(seed)
    hq, hkv, dim, nodes, pool = 8, 2, 64, 9, 64
    lens = [int(x) for x in rng.integers(1, 60, size=3)]
    oracle = CowOracle(pool, hkv, dim)
    planner = PagePool(pool)
    reqs, oreqs = [], []
    for n in lens:  # a base request and a fork of it, per prefix
        pk = U.rand_half(rng, (n, hkv, dim))
        pv = U.rand_half(rng, (n, hkv, dim))
        o = oracle.new(pk, pv)
        r = planner.new(n)
        oreqs += [o, oracle.fork(o)]
        reqs += [r, planner.fork(r)]
    batch = len(reqs)
    draft_q = U.rand_half(rng, (batch, nodes, hq, dim))
    draft_k = U.rand_half(rng, (batch, nodes, hkv, dim))
    draft_v = U.rand_half(rng, (batch, nodes, hkv, dim))
    parent = U.random_tree_parents(rng, batch, nodes)
    paths = []
    for b in range(batch):
        leaf = int(rng.integers(0, nodes))
        path, cur = [], leaf
        while cur >= 0:
            path.append(cur)
            cur = int(parent[b, cur])
        paths.append(path[::-1])
    width = max(len(planner.pages[r]) for r in reqs) + 2
    pages = np.array(planner.page_table(reqs, width), np.int32)
    lengths = np.array([planner.lengths[r] for r in reqs], np.int32)
    plan = planner.plan_commit_batch([(reqs[b], paths[b], b) for b in range(batch)], nodes)
    assert len(plan.clone_src) > 0
    k0, v0 = oracle.k.copy(), oracle.v.copy()
    for b in range(batch):
        oracle.commit(oreqs[b], paths[b], draft_k[b], draft_v[b])
    shape = (batch, hq, hkv, dim, width, pool)
    s = capi.make_shape(*shape)
    t = {"draft_q": U.to_dev(draft_q), "draft_k": U.to_dev(draft_k), "draft_v": U.to_dev(draft_v),
         "parent": U.to_dev(parent), "pages": U.to_dev(pages), "lengths": U.to_dev(lengths)}
    ref_out = torch.empty(batch, nodes, hq, dim, device="cuda")
    capi.tree_verify(s, t["draft_q"], U.to_dev(k0), U.to_dev(v0), t["pages"], t["lengths"],
                     t["draft_k"], t["draft_v"], t["parent"], ref_out, nodes)
    ck, cv = U.to_dev(k0), U.to_dev(v0)
    out = torch.full_like(ref_out, float("nan"))
    capi.last_device_error()
    _fused(capi, s, t, ck, cv, plan, nodes, out)
    torch.cuda.synchronize()
    assert capi.last_device_error() == 0
    assert torch.equal(out, ref_out)
    expected = O.tree(shape, nodes, draft_q, k0, v0, pages, lengths, draft_k, draft_v, parent)
    assert U.max_abs(out.cpu().numpy(), expected) < 2e-4
    assert np.array_equal(U.half_bits(ck), oracle.k)
    assert np.array_equal(U.half_bits(cv), oracle.v)


def test_invalid_entry_leaves_the_clone_its_old_slot(capi):
    """An entry with an out-of-range node writes nothing (and sets the error
    bit); a clone of the page it aimed at must then still receive that
    slot's old contents, as the sequential order (clone, then the entries)
    gives. Through bc_commit_batch, which shares the task code."""
    rng = np.random.default_rng(9)
    hkv, dim, pool, nodes = 2, 64, 6, 3
    k = U.rand_half(rng, (pool, 16, hkv, dim))
    v = U.rand_half(rng, (pool, 16, hkv, dim))
    dk = U.rand_half(rng, (1, nodes, hkv, dim))
    dv = U.rand_half(rng, (1, nodes, hkv, dim))
    ck, cv = U.to_dev(k), U.to_dev(v)
    s = capi.make_shape(1, 4, hkv, dim, 1, pool)
    # clone page 2 -> 4; an in-place entry into page 2 slot 5 with node 7 (bad)
    # and a good one into page 2 slot 6
    capi.last_device_error()
    capi.commit_batch(s, nodes, U.to_dev(dk), U.to_dev(dv), ck, cv, _arr([2]), _arr([4]),
                      _arr([0, 0]), _arr([7, 1]), _arr([2, 2]), _arr([5, 6]))
    torch.cuda.synchronize()
    assert capi.last_device_error() & capi.ERR_COMMIT_INDEX
    ek, ev = k.copy(), v.copy()
    ek[4], ev[4] = k[2], v[2]          # the clone: the whole source page
    ek[2, 6], ev[2, 6] = dk[0, 1], dv[0, 1]  # the valid entry, in place
    assert np.array_equal(U.half_bits(ck), ek)
    assert np.array_equal(U.half_bits(cv), ev)


def test_broken_clone_contract_is_reported(capi):
    """A plan whose clone destination is another clone's source breaks the
    batch contract; the call reports it in the device error word."""
    hkv, dim, pool = 2, 64, 6
    ck = torch.zeros(pool, 16, hkv, dim, device="cuda", dtype=torch.float16)
    cv = torch.zeros_like(ck)
    d = torch.zeros(1, 2, hkv, dim, device="cuda", dtype=torch.float16)
    s = capi.make_shape(1, 4, hkv, dim, 1, pool)
    capi.last_device_error()
    capi.commit_batch(s, 2, d, d, ck, cv, _arr([1, 3]), _arr([3, 5]), None, None, None, None)
    torch.cuda.synchronize()
    assert capi.last_device_error() & capi.ERR_COMMIT_INDEX
