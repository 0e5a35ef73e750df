"""Tree verification through the C ABI: the reference's known answers
(src/main.cu:252-262), random topological trees (BASELINE config 2 style) and
the FP16-output variant."""
import numpy as np
import pytest
import torch

import bc_testutil as U
import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def capi():
    import bc_capi

    return bc_capi


def _run_tree(capi, shape, nodes, f, out_dtype=torch.float32):
    s = capi.make_shape(*shape)
    t = {n: U.to_dev(f[n]) for n in ("draft_q", "k", "v", "pages", "lengths", "draft_k",
                                     "draft_v", "parent")}
    out = torch.full(t["draft_q"].shape, float("nan"), device="cuda", dtype=out_dtype)
    capi.tree_verify(s, t["draft_q"], t["k"], t["v"], t["pages"], t["lengths"], t["draft_k"],
                     t["draft_v"], t["parent"], out, nodes)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("case", range(len(U.TREE_CASES)))
def test_reference_tree_cases(capi, case):
    g = U.golden()
    prefix, d, seed = U.TREE_CASES[case]
    f = O.ref_tree_fixture(2, prefix, 7, d, seed)
    assert U.digest(f["q"], f["k"], f["v"], f["pages"], f["lengths"], f["draft_q"],
                    f["draft_k"], f["draft_v"], f["parent"]) == str(g[f"tree{case}_sha"])
    got = _run_tree(capi, f["shape"].tuple(), 7, f)
    err = U.max_abs(got, g[f"tree{case}_out"])
    assert err <= 3e-4, f"max_abs_error={err}"
    assert capi.last_device_error() == 0


def _tree_fixture(rng, batch, prefix, nodes, hq=32, hkv=8, dim=128, parents="random",
                  pool=None, shared=True):
    f = U.paged_fixture(rng, batch, hq, hkv, dim, [prefix] * batch, pool_pages=pool,
                        shared_prefix=shared)
    f["draft_q"] = U.rand_half(rng, (batch, nodes, hq, dim))
    f["draft_k"] = U.rand_half(rng, (batch, nodes, hkv, dim))
    f["draft_v"] = U.rand_half(rng, (batch, nodes, hkv, dim))
    f["parent"] = (U.random_tree_parents(rng, batch, nodes) if parents == "random"
                   else U.binary_tree_parents(batch, nodes))
    return f


def _oracle_tree(f, nodes):
    return O.tree(f["shape"], nodes, f["draft_q"], f["k"], f["v"], f["pages"], f["lengths"],
                  f["draft_k"], f["draft_v"], f["parent"])


@pytest.mark.parametrize("batch,prefix,nodes,hq,hkv,dim", [
    (8, 2040, 7, 32, 8, 128),   # BASELINE config 2 shape
    (3, 100, 1, 8, 2, 64),
    (2, 0, 19, 8, 8, 64),       # no prefix; 19 nodes spans two draft pages
    (2, 33, 63, 32, 8, 128),    # 63 nodes: 252 rows -> 8 row chunks
    (1, 300, 256, 4, 2, 64),    # the node cap
    (2, 47, 5, 40, 4, 128),     # GQA group 10 (> 8 rows per head)
])
def test_random_trees(capi, batch, prefix, nodes, hq, hkv, dim):
    rng = np.random.default_rng(batch * 1000 + prefix + nodes)
    f = _tree_fixture(rng, batch, prefix, nodes, hq, hkv, dim)
    expected = _oracle_tree(f, nodes)
    got = _run_tree(capi, f["shape"], nodes, f)
    U.assert_close_baseline(got, expected)
    assert U.max_abs(got, expected) < 2e-4


def test_private_prefixes_more_ctas_than_sms(capi):
    """80 requests with private 2040-token prefixes: 4 runs per CTA and 160
    CTAs, more than one wave on 148 SMs. Matches the oracle, and 400 launches
    back to back (programmatic dependent launches, with the softmax groups
    free to run ahead of the PV issuer) leave the device error word clear and
    the output bit-identical (this shape once exposed a barrier-phase
    aliasing stall)."""
    rng = np.random.default_rng(80)
    f = _tree_fixture(rng, 80, 2040, 7, shared=False)
    expected = _oracle_tree(f, 7)
    s = capi.make_shape(*f["shape"])
    t = {n: U.to_dev(f[n]) for n in ("draft_q", "k", "v", "pages", "lengths", "draft_k",
                                     "draft_v", "parent")}
    out = torch.full(t["draft_q"].shape, float("nan"), device="cuda")

    def run():
        capi.tree_verify(s, t["draft_q"], t["k"], t["v"], t["pages"], t["lengths"],
                         t["draft_k"], t["draft_v"], t["parent"], out, 7)

    capi.last_device_error()
    run()
    torch.cuda.synchronize()
    first = out.cpu().numpy()
    U.assert_close_baseline(first, expected)
    assert U.max_abs(first, expected) < 2e-4
    for _ in range(400):
        run()
    torch.cuda.synchronize()
    assert capi.last_device_error() == 0
    assert np.array_equal(out.cpu().numpy(), first)


def test_baseline_config1_fp16_output(capi):
    """1 request, 2048-token prefix in a seeded permutation of a 256-page pool,
    parents [-1,0,0,1,1,2,2], FP16 output checked at the BASELINE tolerance."""
    rng = np.random.default_rng(2048)
    f = _tree_fixture(rng, 1, 2048, 7, pool=256, parents="binary")
    expected = _oracle_tree(f, 7)
    got = _run_tree(capi, f["shape"], 7, f, out_dtype=torch.float16)
    U.assert_close_baseline(got, expected)
    got32 = _run_tree(capi, f["shape"], 7, f)
    U.assert_close_baseline(got32, expected, atol=1e-4, rtol=1e-4)


def test_non_topological_acyclic_parents(capi):
    """The reference walks any acyclic parent chain; so does this kernel."""
    rng = np.random.default_rng(77)
    f = _tree_fixture(rng, 1, 20, 5, 8, 2, 64)
    f["parent"] = np.array([[2, 2, -1, 0, 3]], np.int32)
    expected = _oracle_tree(f, 5)
    got = _run_tree(capi, f["shape"], 5, f)
    assert U.max_abs(got, expected) < 2e-4
    assert capi.last_device_error() == 0


@pytest.mark.parametrize("nodes,hq,hkv", [(7, 32, 8), (3, 8, 8), (20, 16, 2)])
def test_mixed_prefix_runs(capi, nodes, hq, hkv):
    """Requests of one 128-row tile that share a prefix only in runs:
    [A, A, B, C, C, C] (B shares A's pages but not its length; C is disjoint),
    plus an empty prefix at the end."""
    rng = np.random.default_rng(nodes * 31 + hq)
    dim, pool = 64, 90
    perm = rng.permutation(pool).astype(np.int32)
    lens = np.array([300, 300, 290, 517, 517, 517, 0], np.int32)
    batch = len(lens)
    max_pages = 33
    pages = np.full((batch, max_pages), -1, np.int32)
    pages[0, :19] = perm[:19]
    pages[1, :19] = perm[:19]
    pages[2, :19] = perm[:19]
    for b in (3, 4, 5):
        pages[b, :33] = perm[19:52]
    f = dict(shape=(batch, hq, hkv, dim, max_pages, pool), pages=pages, lengths=lens,
             k=U.rand_half(rng, (pool, 16, hkv, dim)), v=U.rand_half(rng, (pool, 16, hkv, dim)),
             draft_q=U.rand_half(rng, (batch, nodes, hq, dim)),
             draft_k=U.rand_half(rng, (batch, nodes, hkv, dim)),
             draft_v=U.rand_half(rng, (batch, nodes, hkv, dim)),
             parent=U.random_tree_parents(rng, batch, nodes))
    expected = _oracle_tree(f, nodes)
    got = _run_tree(capi, f["shape"], nodes, f)
    U.assert_close_baseline(got, expected)
    assert U.max_abs(got, expected) < 2e-4
    assert capi.last_device_error() == 0


@pytest.mark.parametrize("batch,nodes,hq,hkv,dim,out_dtype", [
    (40, 63, 32, 8, 128, torch.float32),   # 252 rows per request: two row tiles
    (40, 63, 32, 8, 128, torch.float16),
    (80, 40, 16, 4, 64, torch.float16),    # 160 rows per request, D = 64
    (80, 40, 16, 4, 64, torch.float32),
])
def test_two_row_tiles_per_cta(capi, batch, nodes, hq, hkv, dim, out_dtype):
    """Requests of more than 128 rows in a grid of several waves: one CTA runs
    both row tiles of a request over each K/V tile. Private prefixes of mixed
    lengths (empty, partial last pages, several tiles) and random trees;
    repeated launches stay bit-identical with the device error word clear."""
    rng = np.random.default_rng(batch * 7 + nodes + dim)
    lens = rng.integers(0, 300, size=batch).astype(np.int32)
    lens[0], lens[1], lens[2] = 0, 64, 1
    f = U.paged_fixture(rng, batch, hq, hkv, dim, lens)
    f["draft_q"] = U.rand_half(rng, (batch, nodes, hq, dim))
    f["draft_k"] = U.rand_half(rng, (batch, nodes, hkv, dim))
    f["draft_v"] = U.rand_half(rng, (batch, nodes, hkv, dim))
    f["parent"] = U.random_tree_parents(rng, batch, nodes)
    expected = _oracle_tree(f, nodes)
    capi.last_device_error()
    got = _run_tree(capi, f["shape"], nodes, f, out_dtype=out_dtype)
    U.assert_close_baseline(got, expected)
    if out_dtype == torch.float32:
        assert U.max_abs(got, expected) < 2e-4
    assert capi.last_device_error() == 0
    s = capi.make_shape(*f["shape"])
    t = {n: U.to_dev(f[n]) for n in ("draft_q", "k", "v", "pages", "lengths", "draft_k",
                                     "draft_v", "parent")}
    out = torch.empty(t["draft_q"].shape, device="cuda", dtype=out_dtype)
    for _ in range(50):
        capi.tree_verify(s, t["draft_q"], t["k"], t["v"], t["pages"], t["lengths"],
                         t["draft_k"], t["draft_v"], t["parent"], out, nodes)
    torch.cuda.synchronize()
    assert capi.last_device_error() == 0
    assert np.array_equal(out.float().cpu().numpy(), got)
