"""Packed-cache decode through the C ABI: the reference's HND/NHD strided
layouts (tests/test_torch_ops.py:62-96 semantics) and vLLM's
[num_blocks, 2, 16, Hkv, D] layout (BASELINE config 4 shape, smaller batch)."""
import math

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


@pytest.mark.parametrize("layout", ["HND", "NHD"])
@pytest.mark.parametrize("dim", [64, 128])
def test_reference_layouts(capi, layout, dim):
    rng = np.random.default_rng(11 + dim)
    batch, hq, hkv, P = 3, 8, 2, 9
    if layout == "HND":
        cache = U.rand_half(rng, (P, hkv, 16, 2 * dim))
        t = U.to_dev(cache)
    else:
        cache_nhd = U.rand_half(rng, (P, 16, hkv, 2 * dim))
        t = U.to_dev(cache_nhd).transpose(1, 2)
        cache = np.ascontiguousarray(cache_nhd)
    q = U.rand_half(rng, (batch, hq, dim))
    pages = np.array([[4, 1], [2, 7], [8, 6]], np.int32)
    lengths = np.array([23, 9, 0], np.int32)
    bs, hs, ss = t.stride(0), t.stride(1), t.stride(2)
    scale = 1 / math.sqrt(dim)
    expected = O.packed_decode((batch, hq, hkv, dim, 2, P), q, cache, pages, lengths,
                               bs, hs, ss, dim, scale)
    s = capi.make_shape(batch, hq, hkv, dim, 2, P)
    dq, dpages, dlengths = U.to_dev(q), U.to_dev(pages), U.to_dev(lengths)
    out = torch.full((batch, hq, dim), float("nan"), device="cuda", dtype=torch.float16)
    capi.packed_decode(s, dq, t, dpages, dlengths, out, bs, hs, ss, scale)
    torch.cuda.synchronize()
    got = O.h2f(U.half_bits(out))
    U.assert_close_baseline(got, O.h2f(expected), atol=1e-3, rtol=1e-3)
    # Same op replayed from a captured CUDA graph (stream correctness).
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        capi.packed_decode(s, dq, t, dpages, dlengths, out, bs, hs, ss, scale)
    out.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    assert np.array_equal(O.h2f(U.half_bits(out)), got)


@pytest.mark.parametrize("splits", [0, 1, 2, 4, 8])
def test_vllm_layout_ragged(capi, splits):
    """[num_blocks, 2, 16, Hkv, D] with seeded non-overlapping block tables and
    ragged lengths; BASELINE tolerance against the oracle."""
    rng = np.random.default_rng(256 + splits)
    batch, hq, hkv, dim = 16, 32, 8, 128
    lengths = rng.integers(512, 8193, size=batch).astype(np.int32)
    lengths[3] = 0
    lengths[5] = 1
    lengths[6] = 17
    npages = (lengths + 15) // 16
    max_pages = int(npages.max())
    nblocks = int(npages.sum()) + 5
    perm = rng.permutation(nblocks).astype(np.int32)
    pages = np.full((batch, max_pages), -1, np.int32)
    cur = 0
    for b in range(batch):
        pages[b, :npages[b]] = perm[cur:cur + npages[b]]
        cur += npages[b]
    cache = U.rand_half(rng, (nblocks, 2, 16, hkv, dim))
    q = U.rand_half(rng, (batch, hq, dim))
    bs, hs, ss, off = 2 * 16 * hkv * dim, dim, hkv * dim, 16 * hkv * dim
    scale = 1 / math.sqrt(dim)
    expected = O.packed_decode((batch, hq, hkv, dim, max_pages, nblocks), q, cache, pages,
                               lengths, bs, hs, ss, off, scale)
    s = capi.make_shape(batch, hq, hkv, dim, max_pages, nblocks)
    out = torch.full((batch, hq, dim), float("nan"), device="cuda", dtype=torch.float16)
    capi.packed_decode_kv(s, U.to_dev(q), U.to_dev(cache), U.to_dev(pages), U.to_dev(lengths),
                          out, bs, hs, ss, off, scale, splits)
    torch.cuda.synchronize()
    got = O.h2f(U.half_bits(out))
    U.assert_close_baseline(got, O.h2f(expected))
    assert U.max_abs(got, O.h2f(expected)) <= 1e-3
    assert capi.last_device_error() == 0


def test_rejects_bad_arguments(capi):
    s = capi.make_shape(1, 8, 2, 64, 1, 4)
    q = torch.zeros(1, 8, 64, device="cuda", dtype=torch.float16)
    cache = torch.zeros(4, 2, 16, 128, device="cuda", dtype=torch.float16)
    pages = torch.zeros(1, 1, device="cuda", dtype=torch.int32)
    lengths = torch.ones(1, device="cuda", dtype=torch.int32)
    out = torch.empty_like(q)
    lib = capi.lib()
    import ctypes

    def call(scale=0.125, bs=4096, hs=2048, ss=128):
        return lib.bc_packed_decode(ctypes.byref(s), capi._ptr(q), capi._ptr(cache),
                                    capi._ptr(pages), capi._ptr(lengths), capi._ptr(out),
                                    bs, hs, ss, scale, capi._stream())

    assert call() == 0
    assert call(scale=0.0) == 1
    assert call(bs=0) == 1
    assert call(ss=3) == 1  # not a 16-byte multiple: the TMA path rejects it
