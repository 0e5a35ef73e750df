"""Parity at BASELINE's own shapes (configs 3, 4, 5a and 5b) against the CPU
oracle.

Inputs are drawn on the GPU from seeded torch generators (N(0,1) FP16, seeded
random physical page permutations) and copied to the host for the oracle, so
multi-gigabyte caches cost seconds rather than minutes of host RNG. The gate is
BASELINE's: max-abs 2e-3 plus relative 1e-2, elementwise; FP32 outputs must
also meet the reference's own 3e-4 max-abs gate (src/main.cu:338).

Reference semantics: decode src/main.cu:81-113 and src/paged_gqa.cu:16-106,
packed decode src/packed_decode.cu:16-61, tree verify src/main.cu:204-240.
"""
import math

import numpy as np
import pytest
import torch

import bc_testutil as U
import oracle as O

pytestmark = pytest.mark.gpu

HQ, HKV, D = 32, 8, 128
SCALE = 1.0 / math.sqrt(D)
REF_GATE = 3e-4  # the reference's own max-abs gate for FP32 outputs


@pytest.fixture(scope="module")
def capi():
    import bc_capi

    return bc_capi


def _gen(seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return g


def _randn(shape, g):
    return torch.randn(shape, generator=g, device="cuda", dtype=torch.float16)


def _release():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


# ---------------------------------------------------------------- config 3
@pytest.fixture(scope="module")
def decode_pool():
    """One K/V pool large enough for 4 x 131,072 tokens; every config-3 shape
    maps its pages to a seeded random subset of it."""
    P = 4 * 131072 // 16 + 8
    g = _gen(3003)
    k, v = _randn((P, 16, HKV, D), g), _randn((P, 16, HKV, D), g)
    pool = {"P": P, "k": k, "v": v, "k_host": U.half_bits(k), "v_host": U.half_bits(v)}
    yield pool
    pool.clear()
    _release()


@pytest.mark.parametrize("batch", [1, 2, 4])
@pytest.mark.parametrize("ctx", [32768, 65536, 131072])
def test_config3_long_context_decode(capi, decode_pool, batch, ctx):
    """batch {1,2,4} x context {32K, 64K, 128K}, one query
    token per request, splits {1, 4, 16, 64} with the FP32 merge."""
    P = decode_pool["P"]
    g = _gen(batch * 1000003 + ctx)
    npg = ctx // 16
    perm = torch.randperm(P, generator=g, device="cuda").to(torch.int32)
    pages = perm[:batch * npg].view(batch, npg).contiguous()
    lengths = torch.full((batch,), ctx, device="cuda", dtype=torch.int32)
    q = _randn((batch, HQ, D), g)
    shape = (batch, HQ, HKV, D, npg, P)
    expected = O.decode(shape, U.half_bits(q), decode_pool["k_host"], decode_pool["v_host"],
                        pages.cpu().numpy(), lengths.cpu().numpy())
    s = capi.make_shape(*shape)
    rows = batch * HQ
    capi.last_device_error()
    for splits in (1, 4, 16, 64):
        out = torch.full((batch, HQ, D), float("nan"), device="cuda")
        pa = torch.empty(splits * rows * D, device="cuda")
        pml = torch.empty(splits * rows * 2, device="cuda")
        capi.decode(s, q, decode_pool["k"], decode_pool["v"], pages, lengths, out, pa, pml,
                    splits)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        U.assert_close_baseline(got, expected)
        err = U.max_abs(got, expected)
        assert err <= REF_GATE, f"splits={splits} max_abs_error={err}"
    # the auto split count and the cluster-merged entry point on the same inputs
    out = torch.full((batch, HQ, D), float("nan"), device="cuda")
    capi.paged_decode(s, q, decode_pool["k"], decode_pool["v"], pages, lengths, out, 0)
    torch.cuda.synchronize()
    assert U.max_abs(out.cpu().numpy(), expected) <= REF_GATE
    assert capi.last_device_error() == 0


# ---------------------------------------------------------------- config 4
def test_config4_packed_decode_batch256(capi):
    """256 one-token decodes, lengths U[512, 8192] from a
    seed, vLLM's [num_blocks, 2, 16, 8, 128] cache (4.6 GB: element offsets
    beyond 2^31) with seeded non-overlapping block tables; FP16 output."""
    rng = np.random.default_rng(256)
    batch = 256
    lengths = rng.integers(512, 8193, size=batch).astype(np.int32)
    npg = (lengths + 15) // 16
    nb, mp = int(npg.sum()), int(npg.max())
    perm = rng.permutation(nb).astype(np.int32)
    pages = np.full((batch, mp), -1, np.int32)
    cur = 0
    for b in range(batch):
        pages[b, :npg[b]] = perm[cur:cur + npg[b]]
        cur += npg[b]
    g = _gen(4004)
    cache = _randn((nb, 2, 16, HKV, D), g)
    assert cache.numel() > 2 ** 31
    q = _randn((batch, HQ, D), g)
    bs, hs, ss, off = 2 * 16 * HKV * D, D, HKV * D, 16 * HKV * D
    shape = (batch, HQ, HKV, D, mp, nb)
    expected = O.h2f(O.packed_decode(shape, U.half_bits(q), U.half_bits(cache), pages, lengths,
                                     bs, hs, ss, off, SCALE))
    s = capi.make_shape(*shape)
    dpages, dlengths = U.to_dev(pages), U.to_dev(lengths)
    capi.last_device_error()
    for splits in (0, 1, 4, 8):
        out = torch.full((batch, HQ, D), float("nan"), device="cuda", dtype=torch.float16)
        capi.packed_decode_kv(s, q, cache, dpages, dlengths, out, bs, hs, ss, off, SCALE, splits)
        torch.cuda.synchronize()
        got = O.h2f(U.half_bits(out))
        U.assert_close_baseline(got, expected)
        assert U.max_abs(got, expected) <= 1e-3, f"splits={splits}"
    assert capi.last_device_error() == 0
    del cache
    _release()


# ---------------------------------------------------------------- config 5a
@pytest.fixture(scope="module")
def tree_scale():
    """BASELINE config 5a inputs: 1024 requests, each a 63-node full binary
    tree over a 4096-token prefix shared by groups of 16 (64 groups, seeded
    page permutation); the oracle's rows for two whole prefix groups (the
    first and a seeded other one), computed once for both output types."""
    total, group, prefix, nodes = 1024, 16, 4096, 63
    ngroups, npg = total // group, prefix // 16
    P = ngroups * npg + 8
    g = _gen(5005)
    k, v = _randn((P, 16, HKV, D), g), _randn((P, 16, HKV, D), g)
    perm = torch.randperm(P, generator=g, device="cuda").to(torch.int32)
    gp = perm[:ngroups * npg].view(ngroups, npg)
    t = dict(total=total, group=group, nodes=nodes, npg=npg, P=P, k=k, v=v,
             pages=gp.repeat_interleave(group, dim=0).contiguous(),
             lengths=torch.full((total,), prefix, device="cuda", dtype=torch.int32),
             dq=_randn((total, nodes, HQ, D), g), dk=_randn((total, nodes, HKV, D), g),
             dv=_randn((total, nodes, HKV, D), g),
             parent=torch.tensor([[-1] + [(n - 1) // 2 for n in range(1, nodes)]] * total,
                                 device="cuda", dtype=torch.int32))
    other = int(np.random.default_rng(55).integers(1, ngroups))
    t["expected"] = {}
    local = np.tile(np.arange(npg, dtype=np.int32), (group, 1))
    for grp in (0, other):
        reqs = slice(grp * group, (grp + 1) * group)
        ids = gp[grp].long()
        t["expected"][grp] = O.tree(
            (group, HQ, HKV, D, npg, npg), nodes, U.half_bits(t["dq"][reqs]),
            U.half_bits(k[ids]), U.half_bits(v[ids]), local, np.full(group, prefix, np.int32),
            U.half_bits(t["dk"][reqs]), U.half_bits(t["dv"][reqs]),
            t["parent"][reqs].cpu().numpy())
    yield t
    t.clear()
    _release()


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_config5a_full_launch(capi, tree_scale, out_dtype):
    """Config 5a as one launch (FP16 output as the bench runs it, FP32 as the
    reference API returns it); every row of the two oracle groups checked."""
    t = tree_scale
    out = torch.full((t["total"], t["nodes"], HQ, D), float("nan"), device="cuda",
                     dtype=out_dtype)
    s = capi.make_shape(t["total"], HQ, HKV, D, t["npg"], t["P"])
    capi.last_device_error()
    capi.tree_verify(s, t["dq"], t["k"], t["v"], t["pages"], t["lengths"], t["dk"], t["dv"],
                     t["parent"], out, t["nodes"])
    torch.cuda.synchronize()
    assert capi.last_device_error() == 0
    for grp, expected in t["expected"].items():
        got = out[grp * t["group"]:(grp + 1) * t["group"]].float().cpu().numpy()
        U.assert_close_baseline(got, expected)
        if out_dtype == torch.float32:
            err = U.max_abs(got, expected)
            assert err <= REF_GATE, f"group {grp}: max_abs_error={err}"
    del out
    _release()


# ---------------------------------------------------------------- config 5b
@pytest.fixture(scope="module")
def million_context():
    """One request of 1,048,576 tokens (65,536 pages, 2 GiB each of K and V:
    byte offsets beyond 2^31) in a seeded page permutation."""
    tokens = 1 << 20
    npg = tokens // 16
    P = npg + 8
    g = _gen(7007)
    k, v = _randn((P, 16, HKV, D), g), _randn((P, 16, HKV, D), g)
    pages = torch.randperm(P, generator=g, device="cuda").to(torch.int32)[:npg].view(1, npg)
    q = _randn((1, HQ, D), g)
    lengths = torch.tensor([tokens], device="cuda", dtype=torch.int32)
    expected = O.decode((1, HQ, HKV, D, npg, P), U.half_bits(q), U.half_bits(k), U.half_bits(v),
                        pages.cpu().numpy(), lengths.cpu().numpy())
    ctx = dict(tokens=tokens, npg=npg, P=P, k=k, v=v, pages=pages.contiguous(), q=q,
               lengths=lengths, expected=expected)
    yield ctx
    ctx.clear()
    _release()


def test_config5b_one_gpu_decode(capi, million_context):
    """The whole 1M-token context on one GPU: 64 global splits and the merge."""
    c = million_context
    s = capi.make_shape(1, HQ, HKV, D, c["npg"], c["P"])
    out = torch.full((1, HQ, D), float("nan"), device="cuda")
    pa = torch.empty(64 * HQ * D, device="cuda")
    pml = torch.empty(64 * HQ * 2, device="cuda")
    capi.last_device_error()
    capi.decode(s, c["q"], c["k"], c["v"], c["pages"], c["lengths"], out, pa, pml, 64)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    U.assert_close_baseline(got, c["expected"])
    assert U.max_abs(got, c["expected"]) <= REF_GATE
    assert capi.last_device_error() == 0


@pytest.mark.parametrize("world", [2, 8])
@pytest.mark.parametrize("reduce_local", [False, True])
def test_config5b_split_across_emulated_ranks(capi, million_context, world, reduce_local):
    """The 1M-token context split into `world` contiguous page shards, one
    bc_paged_decode_partial per shard (37 splits per q-head, as the bench runs
    it). reduce_local: each shard's splits reduced to one partial per row by
    bc_merge_to_partial (what a rank sends in the bench); otherwise all 37
    are sent. The per-rank buffers are stacked as the all-gather delivers them
    and reduced by one bc_merge_gathered."""
    from bc_dist import block_floats, block_views, shard_pages

    c = million_context
    splits = 37
    sent = 1 if reduce_local else splits
    blocks = []
    capi.last_device_error()
    for r in range(world):
        shard = shard_pages(c["npg"], world, r)
        pages = c["pages"][:, shard.start:shard.stop].contiguous()
        length = torch.tensor([len(shard) * 16], device="cuda", dtype=torch.int32)
        s = capi.make_shape(1, HQ, HKV, D, len(shard), c["P"])
        part = torch.full((block_floats(splits, HQ, D),), float("nan"), device="cuda")
        pml, pa = block_views(part, splits, HQ, D)
        capi.paged_decode_partial(s, c["q"], c["k"], c["v"], pages, length, pml, pa, splits)
        if reduce_local:
            buf = torch.full((block_floats(1, HQ, D),), float("nan"), device="cuda")
            ml1, a1 = block_views(buf, 1, HQ, D)
            capi.merge_to_partial(pml, pa, ml1[0], a1[0])
            blocks.append(buf)
        else:
            blocks.append(part)
    out = torch.full((HQ, D), float("nan"), device="cuda")
    capi.merge_gathered(torch.stack(blocks), world, sent, HQ, D, out)
    torch.cuda.synchronize()
    got = out.view(1, HQ, D).cpu().numpy()
    U.assert_close_baseline(got, c["expected"])
    assert U.max_abs(got, c["expected"]) <= REF_GATE
    assert capi.last_device_error() == 0
