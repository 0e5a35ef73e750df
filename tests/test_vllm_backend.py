"""The vLLM V1 backend boundary (reference python/branchcraft_vllm/backend.py,
tests/test_vllm_backend.py): which calls take the Branchcraft fast path, that
every other call reaches TritonAttentionImpl.forward untouched, and (on the
GPU) that the fast path's output equals the oracle's packed decode for both
cache layouts, through a captured CUDA graph too.

The guard tests run on CPU tensors: the guard reads only shapes, strides,
dtypes and metadata fields, and launches nothing.
"""
import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import bc_testutil as U
import oracle as O

pytest.importorskip("vllm")
from vllm.v1.attention.backend import AttentionType  # noqa: E402
from vllm.v1.attention.backends.triton_attn import (  # noqa: E402
    TritonAttentionBackend,
    TritonAttentionImpl,
)

from branchcraft_vllm import backend as B  # noqa: E402


def _impl(hq=4, hkv=2, d=64, **kw):
    return B.BranchcraftImpl(hq, d, 1 / math.sqrt(d), hkv, kw.pop("alibi", None),
                             kw.pop("window", None), kw.pop("kv_dtype", "auto"), **kw)


def _metadata(pages, lengths, max_query_len=1, **extra):
    """The fields the installed vLLM's TritonAttentionMetadata carries for the
    guard (no `causal` / `rswa_window`: vLLM 0.22 has neither)."""
    n = lengths.shape[0]
    md = SimpleNamespace(
        num_actual_tokens=n, max_query_len=max_query_len,
        query_start_loc=torch.arange(n + 1, dtype=torch.int32, device=lengths.device),
        use_cascade=False, mm_prefix_range_tensor=None,
        block_table=pages, seq_lens=lengths)
    for k, v in extra.items():
        setattr(md, k, v)
    return md


def _planes_cache(blocks, hkv, d, device="cpu", gen=None):
    shape = TritonAttentionBackend.get_kv_cache_shape(blocks, 16, hkv, d)
    return torch.randn(shape, dtype=torch.float16, device=device, generator=gen)


def _interleaved_cache(blocks, hkv, d, device="cpu", gen=None):
    # physical [P, 16, Hkv, 2D], logical [P, Hkv, 16, 2D] (the reference test's NHD case)
    return torch.randn(blocks, 16, hkv, 2 * d, dtype=torch.float16, device=device,
                       generator=gen).transpose(1, 2)


def _call(hq=4, hkv=2, d=64, layout="planes"):
    n = 2
    q = torch.randn(n, hq, d, dtype=torch.float16)
    cache = (_planes_cache if layout == "planes" else _interleaved_cache)(6, hkv, d)
    pages = torch.tensor([[3, 1], [4, 2]], dtype=torch.int32)
    lengths = torch.tensor([19, 7], dtype=torch.int32)
    out = torch.empty(n, hq * d, dtype=torch.float16)
    return q, cache, _metadata(pages, lengths), out


# ------------------------------------------------------------------ guard


@pytest.mark.parametrize("layout,kind", [("planes", B.PLANES), ("interleaved", B.INTERLEAVED)])
def test_guard_accepts_one_token_decode(layout, kind):
    impl = _impl()
    q, cache, md, out = _call(layout=layout)
    assert impl._decode_layout(q, cache, md, out, None, None) == kind
    assert impl._can_decode(q, cache, md, out, None, None)


def _mutations():
    """(name, function(impl, q, cache, md, out) -> args) each of which must
    send the call to the Triton fallback."""
    def impl_attr(**kv):
        def f(impl, q, cache, md, out):
            for k, v in kv.items():
                setattr(impl, k, v)
            return q, cache, md, out, None, None
        return f

    def md_attr(**kv):
        def f(impl, q, cache, md, out):
            for k, v in kv.items():
                setattr(md, k, v)
            return q, cache, md, out, None, None
        return f

    return [
        ("prefill", md_attr(max_query_len=2)),
        ("no metadata", lambda i, q, c, m, o: (q, c, None, o, None, None)),
        ("no tokens", md_attr(num_actual_tokens=0)),
        ("ragged query_start_loc", md_attr(query_start_loc=torch.tensor([0, 2], dtype=torch.int32))),
        ("non-causal", md_attr(causal=False)),
        ("cascade", md_attr(use_cascade=True)),
        ("multimodal prefix", md_attr(mm_prefix_range_tensor=torch.zeros(2, 1, 2))),
        ("ragged window", md_attr(rswa_window=128)),
        ("encoder", impl_attr(attn_type=AttentionType.ENCODER)),
        ("sliding window", impl_attr(sliding_window=(127, 0))),
        ("alibi", impl_attr(alibi_slopes=torch.ones(4))),
        ("sinks", impl_attr(sinks=torch.zeros(4))),
        ("soft cap", impl_attr(logits_soft_cap=30.0)),
        ("fp8 cache dtype", impl_attr(kv_cache_dtype="fp8")),
        ("per-token-head quant", impl_attr(_is_per_token_head_quant=True)),
        ("chunk lookback", impl_attr(chunk_lookback=64)),
        ("bf16 query", lambda i, q, c, m, o: (q.bfloat16(), c, m, o, None, None)),
        ("bf16 cache", lambda i, q, c, m, o: (q, c.bfloat16(), m, o, None, None)),
        ("fp32 output", lambda i, q, c, m, o: (q, c, m, o.float(), None, None)),
        ("strided query", lambda i, q, c, m, o: (q.transpose(0, 1).contiguous().transpose(0, 1),
                                                 c, m, o, None, None)),
        ("output scale", lambda i, q, c, m, o: (q, c, m, o, torch.ones(1), None)),
        ("output block scale", lambda i, q, c, m, o: (q, c, m, o, None, torch.ones(1))),
        ("int64 block table", md_attr(block_table=torch.tensor([[3, 1], [4, 2]]))),
        ("int64 seq_lens", md_attr(seq_lens=torch.tensor([19, 7]))),
        ("strided block table", md_attr(
            block_table=torch.tensor([[3, 0, 1, 0], [4, 0, 2, 0]], dtype=torch.int32)[:, ::2])),
        ("block size 32", lambda i, q, c, m, o: (
            q, torch.zeros(3, 2, 32, 2, 64, dtype=torch.float16), m, o, None, None)),
        ("head-size mismatch", lambda i, q, c, m, o: (
            q, torch.zeros(6, 2, 16, 2, 128, dtype=torch.float16), m, o, None, None)),
        ("kv-head mismatch", lambda i, q, c, m, o: (
            q, torch.zeros(6, 2, 16, 4, 64, dtype=torch.float16), m, o, None, None)),
        ("strided head dim", lambda i, q, c, m, o: (
            q, torch.zeros(6, 2, 16, 2, 128, dtype=torch.float16)[..., ::2], m, o, None, None)),
    ]


@pytest.mark.parametrize("name,mutate", _mutations(), ids=[m[0] for m in _mutations()])
def test_guard_falls_back(name, mutate):
    impl = _impl()
    q, cache, md, out = _call()
    args = mutate(impl, q, cache, md, out)
    assert not impl._can_decode(*args), name


def test_guard_rejects_unsupported_head_size():
    impl = _impl(hq=4, hkv=2, d=96)
    q = torch.zeros(2, 4, 96, dtype=torch.float16)
    cache = torch.zeros(6, 2, 16, 2, 96, dtype=torch.float16)
    md = _metadata(torch.zeros(2, 2, dtype=torch.int32), torch.ones(2, dtype=torch.int32))
    assert not impl._can_decode(q, cache, md, torch.zeros(2, 4 * 96, dtype=torch.float16),
                                None, None)


def test_fallback_reaches_triton_forward(monkeypatch, capsys):
    """A prefill call goes to TritonAttentionImpl.forward with every argument
    unchanged, and the trace line is printed once."""
    seen = []

    def fake_forward(self, layer, query, key, value, kv_cache, md, output, output_scale=None,
                     output_block_scale=None):
        seen.append((layer, query, key, value, kv_cache, md, output, output_scale,
                     output_block_scale))
        return output

    monkeypatch.setattr(TritonAttentionImpl, "forward", fake_forward)
    monkeypatch.setenv("BRANCHCRAFT_TRACE", "1")
    monkeypatch.setattr(B.BranchcraftImpl, "_reported_prefill_fallback", False)
    impl = _impl()
    q, cache, md, out = _call()
    md.max_query_len = 2
    layer = object()
    for _ in range(2):
        assert impl.forward(layer, q, q, q, cache, md, out) is out
    assert len(seen) == 2 and seen[0][0] is layer and seen[0][4] is cache and seen[0][6] is out
    assert capsys.readouterr().out.count("BRANCHCRAFT_PREFILL_FALLBACK TritonAttentionImpl") == 1


def test_backend_class_and_plugin():
    from vllm.v1.attention.backends.registry import AttentionBackendEnum

    from branchcraft_vllm import plugin

    assert B.BranchcraftBackend.get_name() == "CUSTOM"
    assert B.BranchcraftBackend.get_impl_cls() is B.BranchcraftImpl
    was = AttentionBackendEnum.CUSTOM.is_overridden()
    try:
        plugin.register()
        assert AttentionBackendEnum.CUSTOM.get_class() is B.BranchcraftBackend
    finally:
        if not was:
            AttentionBackendEnum.CUSTOM.clear_override()


# ------------------------------------------------------------------ GPU


def _oracle_for(cache, q, pages, lengths, scale, layout):
    """Oracle packed decode over the cache's own strides (elements)."""
    P, d = cache.shape[0], q.shape[2]
    if layout == "planes":
        bs, ss, hs, kv_off = cache.stride(0), cache.stride(2), cache.stride(3), cache.stride(1)
    else:
        bs, hs, ss, kv_off = cache.stride(0), cache.stride(1), cache.stride(2), d
    host = U.half_bits(cache.as_strided((cache.untyped_storage().nbytes() // 2,), (1,)))
    b, hq = q.shape[0], q.shape[1]
    shape = (b, hq, cache.shape[3] if layout == "planes" else cache.shape[1], d,
             pages.shape[1], P)
    return O.packed_decode(shape, U.half_bits(q), host, pages.cpu().numpy(),
                           lengths.cpu().numpy(), bs, hs, ss, kv_off, scale)


def _torch_reference(cache, q, pages, lengths, scale, layout):
    """fp32 torch restatement of the reference test's expected value
    (tests/test_vllm_backend.py:40-49): softmax(K q * scale) V per head."""
    n, hq, d = q.shape
    kc, vc = ((cache[:, 0], cache[:, 1]) if layout == "planes"
              else (cache[..., :d].transpose(1, 2), cache[..., d:].transpose(1, 2)))
    hkv = kc.shape[2]
    kh = torch.arange(hq, device=q.device) // (hq // hkv)
    out = torch.zeros(n, hq, d, device=q.device)
    for b in range(n):
        tok = torch.arange(int(lengths[b]), device=q.device)
        blk = pages[b, tok // 16].long()
        k = kc[blk, tok % 16].float()[:, kh]      # [len, Hq, D]
        v = vc[blk, tok % 16].float()[:, kh]
        s = torch.einsum("hd,thd->ht", q[b].float(), k) * scale
        out[b] = torch.einsum("ht,thd->hd", torch.softmax(s, 1), v)
    return out


@pytest.mark.parametrize("layout", ["planes", "interleaved"])
def test_oracle_strides_match_torch_reference(layout):
    """The oracle call this file's GPU test checks against, given the cache's
    own strides, agrees with the fp32 torch restatement (CPU only)."""
    gen = torch.Generator()
    gen.manual_seed(5)
    cache = (_planes_cache if layout == "planes" else _interleaved_cache)(6, 2, 64, gen=gen)
    q = torch.randn(3, 4, 64, dtype=torch.float16, generator=gen)
    pages = torch.tensor([[3, 1], [4, 2], [5, 0]], dtype=torch.int32)
    lengths = torch.tensor([19, 7, 32], dtype=torch.int32)
    got = O.h2f(_oracle_for(cache, q, pages, lengths, 0.125, layout))
    ref = _torch_reference(cache, q, pages, lengths, 0.125, layout).numpy()
    U.assert_close_baseline(got, ref, atol=2e-3, rtol=1e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["planes", "interleaved"])
@pytest.mark.parametrize("hq,hkv,d", [(4, 2, 64), (32, 8, 128)])
def test_fast_path_matches_oracle(layout, hq, hkv, d, monkeypatch, capsys):
    gen = torch.Generator(device="cuda")
    gen.manual_seed(23 + d + hq)
    rng = np.random.default_rng(7 + d)
    lens = np.array([19, 7, 1, 16, 130, 64], np.int32)
    npg = (lens + 15) // 16
    blocks = int(npg.sum()) + 3
    perm = rng.permutation(blocks).astype(np.int32)
    width = int(npg.max()) + 2
    table = np.zeros((len(lens), width), np.int32)  # vLLM pads rows with block 0
    cur = 0
    for i, k in enumerate(npg):
        table[i, :k] = perm[cur:cur + k]
        cur += k
    make = _planes_cache if layout == "planes" else _interleaved_cache
    cache = make(blocks, hkv, d, "cuda", gen)
    n = len(lens)
    q = torch.randn(n, hq, d, device="cuda", dtype=torch.float16, generator=gen)
    pages = torch.from_numpy(table).cuda()
    lengths = torch.from_numpy(lens).cuda()
    md = _metadata(pages, lengths)
    impl = _impl(hq=hq, hkv=hkv, d=d)
    out = torch.full((n, hq * d), float("nan"), device="cuda", dtype=torch.float16)
    monkeypatch.setenv("BRANCHCRAFT_TRACE", "1")
    monkeypatch.setattr(B.BranchcraftImpl, "_reported_fast_path", False)
    assert impl.forward(None, q, q, q, cache, md, out) is out
    torch.cuda.synchronize()
    kind = B.PLANES if layout == "planes" else B.INTERLEAVED
    assert f"BRANCHCRAFT_FAST_PATH {kind}" in capsys.readouterr().out
    expected = _oracle_for(cache, q, pages, lengths, impl.scale, layout)
    got = U.half_bits(out.view(n, hq, d))
    U.assert_close_baseline(O.h2f(got), O.h2f(expected), atol=2e-3, rtol=1e-2)

    ref = _torch_reference(cache, q, pages, lengths, impl.scale, layout)
    torch.testing.assert_close(out.view(n, hq, d).float(), ref, atol=6e-3, rtol=6e-3)

    # the fast path replays from a captured CUDA graph (vLLM full-graph mode)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        impl.forward(None, q, q, q, cache, md, out)
    out.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    assert np.array_equal(U.half_bits(out.view(n, hq, d)), got)
