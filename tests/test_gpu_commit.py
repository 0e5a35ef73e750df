"""Accepted-path commit and copy-on-write: exact placement (the reference's
test_commit_isolation), the shared-partial-page scenario of src/main.cu:264-313
and a batched commit checked bit-exact against the oracle."""
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


def test_commit_isolation(capi):
    cache_k = torch.zeros(4, 16, 2, 64, device="cuda", dtype=torch.float16)
    cache_v = torch.zeros_like(cache_k)
    draft_k = torch.arange(3, device="cuda", dtype=torch.float16).view(1, 3, 1, 1).expand(
        1, 3, 2, 64).contiguous()
    draft_v = draft_k + 10
    path = torch.tensor([0, 2], device="cuda", dtype=torch.int32)
    dp = torch.tensor([3, 3], device="cuda", dtype=torch.int32)
    ds = torch.tensor([6, 7], device="cuda", dtype=torch.int32)
    s = capi.make_shape(1, 2, 2, 64, 1, 4)
    capi.commit_path(s, draft_k, draft_v, cache_k, cache_v, path, dp, ds, 0, 3, 2)
    torch.cuda.synchronize()
    assert torch.equal(cache_k[3, 6], draft_k[0, 0])
    assert torch.equal(cache_k[3, 7], draft_k[0, 2])
    assert torch.equal(cache_v[3, 7], draft_v[0, 2])
    assert torch.count_nonzero(cache_k[:3]) == 0
    assert torch.count_nonzero(cache_k[3, 8:]) == 0
    assert capi.last_device_error() == 0


def test_shared_page_commit_sibling_rollback(capi):
    """src/main.cu:264-313: clone a shared partial page, commit path {0,1,3}
    to slots 1..3, then decode: accepted == tree output of node 3, sibling and
    rollback unchanged (1e-7)."""
    f = O.ref_tree_fixture(2, 17, 7, 128, 49)
    sh = f["shape"].tuple()
    s = capi.make_shape(*sh)
    t = {n: U.to_dev(f[n]) for n in ("q", "k", "v", "pages", "lengths", "draft_q", "draft_k",
                                     "draft_v", "parent")}
    tree_out = torch.empty(t["draft_q"].shape, device="cuda")
    capi.tree_verify(s, t["draft_q"], t["k"], t["v"], t["pages"], t["lengths"], t["draft_k"],
                     t["draft_v"], t["parent"], tree_out, 7)
    out = torch.empty(2, 32, 128, device="cuda")
    capi.decode(s, t["q"], t["k"], t["v"], t["pages"], t["lengths"], out)
    before = out.clone()
    new_page, old_page = sh[5] - 1, int(f["pages"][0, 1])
    t["k"][new_page].copy_(t["k"][old_page])
    t["v"][new_page].copy_(t["v"][old_page])
    path = torch.tensor([0, 1, 3], device="cuda", dtype=torch.int32)
    dp = torch.full((3,), new_page, device="cuda", dtype=torch.int32)
    ds = torch.tensor([1, 2, 3], device="cuda", dtype=torch.int32)
    capi.commit_path(s, t["draft_k"], t["draft_v"], t["k"], t["v"], path, dp, ds, 0, 7, 3)
    pages2 = f["pages"].copy()
    pages2[0, 1] = new_page
    lengths2 = f["lengths"].copy()
    lengths2[0] += 3
    q2 = t["q"].clone()
    q2[0] = t["draft_q"][0, 3]
    capi.decode(s, q2, t["k"], t["v"], U.to_dev(pages2), U.to_dev(lengths2), out)
    torch.cuda.synchronize()
    accepted = (out[0] - tree_out[0, 3]).abs().max().item()
    sibling = (out[1] - before[1]).abs().max().item()
    assert accepted <= 3e-4 and sibling <= 1e-7
    capi.decode(s, t["q"], t["k"], t["v"], t["pages"], t["lengths"], out)
    torch.cuda.synchronize()
    assert (out - before).abs().max().item() <= 1e-7
    assert capi.last_device_error() == 0


def test_commit_batch_bit_exact(capi):
    rng = np.random.default_rng(3)
    P, hkv, dim, B, N = 40, 8, 128, 4, 7
    ck = U.rand_half(rng, (P, 16, hkv, dim))
    cv = U.rand_half(rng, (P, 16, hkv, dim))
    dk = U.rand_half(rng, (B, N, hkv, dim))
    dv = U.rand_half(rng, (B, N, hkv, dim))
    clone_src = np.array([5, 5, 9], np.int32)
    clone_dst = np.array([30, 31, 32], np.int32)
    req = np.array([0, 0, 1, 2, 2, 2, 3], np.int32)
    node = np.array([0, 3, 0, 0, 1, 4, 6], np.int32)
    page = np.array([30, 30, 31, 5, 5, 33, 32], np.int32)
    slot = np.array([8, 9, 8, 8, 9, 0, 15], np.int32)
    exp_k, exp_v = ck.copy(), cv.copy()
    for a, b in zip(clone_src, clone_dst):
        exp_k[b] = exp_k[a]
        exp_v[b] = exp_v[a]
    for e in range(len(req)):
        O.commit(exp_k, exp_v, dk, dv, node[e:e + 1], page[e:e + 1], slot[e:e + 1], int(req[e]))
    tk, tv = U.to_dev(ck), U.to_dev(cv)
    s = capi.make_shape(B, hkv, hkv, dim, 1, P)
    capi.commit_batch(s, N, U.to_dev(dk), U.to_dev(dv), tk, tv, U.to_dev(clone_src),
                      U.to_dev(clone_dst), U.to_dev(req), U.to_dev(node), U.to_dev(page),
                      U.to_dev(slot))
    torch.cuda.synchronize()
    assert np.array_equal(U.half_bits(tk), exp_k)
    assert np.array_equal(U.half_bits(tv), exp_v)
    assert capi.last_device_error() == 0


def test_commit_batch_many_clones(capi):
    """300 clones of one page (beyond the one-launch limit of 256: every clone,
    then every row commit), an in-place commit into the cloned page and rows
    into some of the clones; bit-exact against clones-first, then commits."""
    rng = np.random.default_rng(5)
    P, hkv, dim, B, N = 320, 2, 64, 4, 3
    ck = U.rand_half(rng, (P, 16, hkv, dim))
    cv = U.rand_half(rng, (P, 16, hkv, dim))
    dk = U.rand_half(rng, (B, N, hkv, dim))
    dv = U.rand_half(rng, (B, N, hkv, dim))
    clone_src = np.full(300, 7, np.int32)
    clone_dst = np.arange(10, 310, dtype=np.int32)
    req = np.array([0, 1, 2, 3], np.int32)
    node = np.array([0, 1, 2, 0], np.int32)
    page = np.array([7, 10, 11, 309], np.int32)
    slot = np.array([8, 8, 9, 15], np.int32)
    exp_k, exp_v = ck.copy(), cv.copy()
    for a, b in zip(clone_src, clone_dst):
        exp_k[b] = exp_k[a]
        exp_v[b] = exp_v[a]
    for e in range(len(req)):
        O.commit(exp_k, exp_v, dk, dv, node[e:e + 1], page[e:e + 1], slot[e:e + 1], int(req[e]))
    tk, tv = U.to_dev(ck), U.to_dev(cv)
    s = capi.make_shape(B, hkv, hkv, dim, 1, P)
    capi.commit_batch(s, N, U.to_dev(dk), U.to_dev(dv), tk, tv, U.to_dev(clone_src),
                      U.to_dev(clone_dst), U.to_dev(req), U.to_dev(node), U.to_dev(page),
                      U.to_dev(slot))
    torch.cuda.synchronize()
    assert np.array_equal(U.half_bits(tk), exp_k)
    assert np.array_equal(U.half_bits(tv), exp_v)
    assert capi.last_device_error() == 0
