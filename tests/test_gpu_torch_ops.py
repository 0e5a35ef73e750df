"""torch.ops.branchcraft at the dispatcher boundary: the reference's own op
tests restated (tests/test_torch_ops.py: tree mask + torch.compile + opcheck,
packed HND/NHD decode + CUDA graph replay, exact commit placement) and the
added ops (paged_decode, tree_verify_out, packed_decode_kv_out, commit_batch_)."""
import math

import numpy as np
import pytest
import torch

import bc_testutil as U
import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bc():
    import branchcraft_torch

    return branchcraft_torch


def _torch_tree_reference(q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent):
    batch, nodes, hq, dim = q.shape
    hkv = prefix_k.shape[2]
    expected = torch.empty(q.shape, device=q.device, dtype=torch.float32)
    for b in range(batch):
        for node in range(nodes):
            path, cur = [], node
            while cur >= 0:
                path.append(cur)
                cur = int(parent[b, cur])
            path.reverse()
            for h in range(hq):
                kvh = h // (hq // hkv)
                keys, vals = [], []
                for t in range(int(lengths[b])):
                    page = int(pages[b, t // 16])
                    keys.append(prefix_k[page, t % 16, kvh].float())
                    vals.append(prefix_v[page, t % 16, kvh].float())
                keys += [draft_k[b, p, kvh].float() for p in path]
                vals += [draft_v[b, p, kvh].float() for p in path]
                scores = torch.stack(keys) @ q[b, node, h].float() / math.sqrt(dim)
                expected[b, node, h] = torch.softmax(scores, 0) @ torch.stack(vals)
    return expected


@pytest.mark.parametrize("dim", [64, 128])
def test_tree_mask_and_compile(bc, dim):
    torch.manual_seed(7)
    batch, nodes, hq, hkv = 2, 7, 4, 2
    q = torch.randn(batch, nodes, hq, dim, device="cuda", dtype=torch.float16)
    prefix_k = torch.randn(7, 16, hkv, dim, device="cuda", dtype=torch.float16)
    prefix_v = torch.randn_like(prefix_k)
    pages = torch.tensor([[4, 1], [5, 2]], device="cuda", dtype=torch.int32)
    lengths = torch.tensor([23, 0], device="cuda", dtype=torch.int32)
    draft_k = torch.randn(batch, nodes, hkv, dim, device="cuda", dtype=torch.float16)
    draft_v = torch.randn_like(draft_k)
    parent = torch.tensor([[-1, 0, 0, 1, 1, 2, 2]] * batch, device="cuda", dtype=torch.int32)
    args = (q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent)
    actual = bc.tree_verify(*args)
    torch.testing.assert_close(actual, _torch_tree_reference(*args), atol=4e-3, rtol=4e-3)
    compiled = torch.compile(bc.tree_verify, backend="inductor")
    torch.testing.assert_close(compiled(*args), actual)
    torch.library.opcheck(torch.ops.branchcraft.tree_verify, args,
                          test_utils=("test_schema", "test_faketensor"))
    out16 = torch.empty(q.shape, device="cuda", dtype=torch.float16)
    bc.tree_verify_out(*args, out16)
    torch.testing.assert_close(out16.float(), actual, atol=2e-3, rtol=1e-2)


@pytest.mark.parametrize("layout", ["HND", "NHD"])
def test_packed_decode_and_graph(bc, layout):
    torch.manual_seed(11)
    batch, hq, hkv, dim = 3, 8, 2, 64
    if layout == "HND":
        cache = torch.randn(9, hkv, 16, 2 * dim, device="cuda", dtype=torch.float16)
    else:
        cache = torch.randn(9, 16, hkv, 2 * dim, device="cuda", dtype=torch.float16).transpose(1, 2)
    q = torch.randn(batch, hq, dim, device="cuda", dtype=torch.float16)
    pages = torch.tensor([[4, 1], [2, 7], [8, 6]], device="cuda", dtype=torch.int32)
    lengths = torch.tensor([23, 9, 0], device="cuda", dtype=torch.int32)
    out = torch.empty_like(q)
    bc.packed_decode_out(q, cache, pages, lengths, out, 1 / math.sqrt(dim))
    expected = torch.zeros_like(q)
    for b in range(batch):
        for h in range(hq):
            kvh = h // (hq // hkv)
            keys, vals = [], []
            for t in range(int(lengths[b])):
                token = cache[int(pages[b, t // 16]), kvh, t % 16]
                keys.append(token[:dim].float())
                vals.append(token[dim:].float())
            if keys:
                scores = torch.stack(keys) @ q[b, h].float() / math.sqrt(dim)
                expected[b, h] = (torch.softmax(scores, 0) @ torch.stack(vals)).half()
    torch.testing.assert_close(out, expected, atol=6e-3, rtol=6e-3)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        bc.packed_decode_out(q, cache, pages, lengths, out, 1 / math.sqrt(dim))
    out.zero_()
    graph.replay()
    torch.testing.assert_close(out, expected, atol=6e-3, rtol=6e-3)


def test_commit_isolation(bc):
    cache_k = torch.zeros(4, 16, 2, 64, device="cuda", dtype=torch.float16)
    cache_v = torch.zeros_like(cache_k)
    draft_k = torch.arange(3, device="cuda", dtype=torch.float16).view(1, 3, 1, 1).expand(
        1, 3, 2, 64).contiguous()
    draft_v = draft_k + 10
    path = torch.tensor([0, 2], device="cuda", dtype=torch.int32)
    dest_pages = torch.tensor([3, 3], device="cuda", dtype=torch.int32)
    dest_slots = torch.tensor([6, 7], device="cuda", dtype=torch.int32)
    bc.commit_path_(cache_k, cache_v, draft_k, draft_v, path, dest_pages, dest_slots, 0)
    torch.testing.assert_close(cache_k[3, 6], draft_k[0, 0])
    torch.testing.assert_close(cache_k[3, 7], draft_k[0, 2])
    torch.testing.assert_close(cache_v[3, 7], draft_v[0, 2])
    assert torch.count_nonzero(cache_k[:3]) == 0
    assert torch.count_nonzero(cache_k[3, 8:]) == 0


def test_paged_decode_op(bc):
    rng = np.random.default_rng(21)
    f = U.paged_fixture(rng, 3, 16, 4, 128, [900, 5, 4000])
    expected = O.decode(f["shape"], f["q"], f["k"], f["v"], f["pages"], f["lengths"])
    args = [U.to_dev(f[n]) for n in ("q", "k", "v", "pages", "lengths")]
    for splits in (0, 1, 4, 16, 64):
        got = bc.paged_decode(*args, splits=splits)
        torch.cuda.synchronize()
        assert U.max_abs(got.cpu().numpy(), expected) < 1e-4
    torch.library.opcheck(torch.ops.branchcraft.paged_decode, (*args, 0),
                          test_utils=("test_schema", "test_faketensor"))


def test_packed_decode_kv_out_vllm_layout(bc):
    """vLLM 0.22's cache [num_blocks, 2, 16, Hkv, D] passed as two strided views."""
    rng = np.random.default_rng(4)
    batch, hq, hkv, dim, nblocks = 4, 32, 8, 128, 80
    lengths = np.array([700, 1, 0, 333], np.int32)
    npages = (lengths + 15) // 16
    pages = np.zeros((batch, int(npages.max())), np.int32)
    perm = rng.permutation(nblocks).astype(np.int32)
    cur = 0
    for b in range(batch):
        pages[b, :npages[b]] = perm[cur:cur + npages[b]]
        cur += npages[b]
    cache = U.rand_half(rng, (nblocks, 2, 16, hkv, dim))
    q = U.rand_half(rng, (batch, hq, dim))
    expected = O.packed_decode((batch, hq, hkv, dim, pages.shape[1], nblocks), q, cache, pages,
                               lengths, 2 * 16 * hkv * dim, dim, hkv * dim, 16 * hkv * dim,
                               1 / math.sqrt(dim))
    t = U.to_dev(cache)
    k_view = t[:, 0].transpose(1, 2)  # [P, Hkv, 16, D]
    v_view = t[:, 1].transpose(1, 2)
    out = torch.full((batch, hq, dim), float("nan"), device="cuda", dtype=torch.float16)
    bc.packed_decode_kv_out(U.to_dev(q), k_view, v_view, U.to_dev(pages), U.to_dev(lengths),
                            out, 1 / math.sqrt(dim))
    torch.cuda.synchronize()
    U.assert_close_baseline(O.h2f(U.half_bits(out)), O.h2f(expected))
