"""Paged GQA split-KV decode through the C ABI against the reference's own
known answers (src/main.cu:318-352) and the oracle on BASELINE-style inputs."""
import numpy as np
import pytest
import torch

import bc_testutil as U
import oracle as O

pytestmark = pytest.mark.gpu

SPLITS = [1, 2, 4, 8, 16, 64]


@pytest.fixture(scope="module")
def capi():
    import bc_capi

    return bc_capi


def _run_decode(capi, f, splits):
    s = capi.make_shape(*f["shape"].tuple()) if hasattr(f["shape"], "tuple") else capi.make_shape(*f["shape"])
    dq, dk, dv = U.to_dev(f["q"]), U.to_dev(f["k"]), U.to_dev(f["v"])
    pages, lengths = U.to_dev(f["pages"]), U.to_dev(f["lengths"])
    out = torch.full(dq.shape, float("nan"), device="cuda", dtype=torch.float32)
    rows = s.batch * s.query_heads
    pa = torch.empty(max(splits, 1) * rows * s.dim, device="cuda")
    pml = torch.empty(max(splits, 1) * rows * 2, device="cuda")
    capi.decode(s, dq, dk, dv, pages, lengths, out, pa, pml, splits)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("case", range(len(U.DECODE_CASES)))
def test_reference_cases_all_splits(capi, case):
    g = U.golden()
    b, hq, hkv, d, lens = U.DECODE_CASES[case]
    f = O.ref_fixture(b, hq, hkv, d, lens, 17)
    assert U.digest(f["q"], f["k"], f["v"], f["pages"]) == str(g[f"decode{case}_sha"])
    expected = g[f"decode{case}_out"]
    for splits in SPLITS:
        got = _run_decode(capi, f, splits)
        err = U.max_abs(got, expected)
        assert err <= 3e-4, f"splits={splits} max_abs_error={err}"
    assert capi.last_device_error() == 0


def test_rejects_bad_arguments(capi):
    f = O.ref_fixture(1, 8, 2, 64, [17], 17)
    s = capi.make_shape(*f["shape"].tuple())
    dq, dk, dv = U.to_dev(f["q"]), U.to_dev(f["k"]), U.to_dev(f["v"])
    pages, lengths = U.to_dev(f["pages"]), U.to_dev(f["lengths"])
    out = torch.empty(dq.shape, device="cuda")
    bad = capi.make_shape(*f["shape"].tuple())
    bad.dim = 96
    assert capi.decode(bad, dq, dk, dv, pages, lengths, out, None, None, 1, check=False) == 1
    assert capi.decode(s, dq, dk, dv, pages, lengths, out, None, None, 2, check=False) == 1
    assert capi.decode(s, dq, dk, dv, pages, lengths, out, None, None, 65, check=False) == 1
    assert capi.decode(s, dq, dk, dv, pages, lengths, out, None, None, 0, check=False) == 1


@pytest.mark.parametrize("batch,ctx", [(1, 4096), (2, 3000), (4, 1037)])
def test_baseline_style_decode(capi, batch, ctx):
    """N(0,1) inputs, seeded page permutation; BASELINE tolerance vs the oracle."""
    rng = np.random.default_rng(1000 + batch)
    lens = [ctx - (i % 4) * ctx // 8 for i in range(batch)]
    f = U.paged_fixture(rng, batch, 32, 8, 128, lens)
    expected = O.decode(f["shape"], f["q"], f["k"], f["v"], f["pages"], f["lengths"])
    for splits in (1, 4, 16, 64):
        got = _run_decode(capi, f, splits)
        U.assert_close_baseline(got, expected)
        assert U.max_abs(got, expected) < 1e-4


def test_auto_splits_and_paged_decode(capi):
    rng = np.random.default_rng(5)
    f = U.paged_fixture(rng, 3, 16, 4, 64, [700, 0, 1500])
    s = capi.make_shape(*f["shape"])
    expected = O.decode(f["shape"], f["q"], f["k"], f["v"], f["pages"], f["lengths"])
    dq, dk, dv = U.to_dev(f["q"]), U.to_dev(f["k"]), U.to_dev(f["v"])
    pages, lengths = U.to_dev(f["pages"]), U.to_dev(f["lengths"])
    for splits in (0, 1, 2, 8):
        out = torch.full(dq.shape, float("nan"), device="cuda")
        capi.paged_decode(s, dq, dk, dv, pages, lengths, out, splits)
        torch.cuda.synchronize()
        assert U.max_abs(out.cpu().numpy(), expected) < 1e-4
    assert capi.auto_splits(s, 100, 148) == 1
    assert 1 <= capi.auto_splits(s, 131072, 148) <= 64


def test_merge_partials_matches_oracle(capi):
    rng = np.random.default_rng(9)
    S, rows, D = 5, 12, 128
    pml = rng.standard_normal((S, rows, 2)).astype(np.float32)
    pml[..., 1] = np.abs(pml[..., 1]) + 0.1
    pml[2, 3, 0] = -np.inf
    pml[:, 7, 0] = -np.inf  # an all-empty row gives zeros
    pa = rng.standard_normal((S, rows, D)).astype(np.float32)
    expected = O.merge(pml, pa)
    out = torch.empty(rows, D, device="cuda")
    capi.merge_partials(torch.from_numpy(pml).cuda(), torch.from_numpy(pa).cuda(), out)
    torch.cuda.synchronize()
    assert U.max_abs(out.cpu().numpy(), expected) < 1e-5


def test_merge_to_partial_then_merge_matches_oracle(capi):
    """Reducing partials in two stages (two groups each merged to ONE partial
    per row, then those merged) equals the oracle's one-stage merge; an
    all-empty row stays zeros through both stages."""
    rng = np.random.default_rng(19)
    S, rows, D = 6, 10, 128
    pml = rng.standard_normal((S, rows, 2)).astype(np.float32)
    pml[..., 1] = np.abs(pml[..., 1]) + 0.1
    pml[:, 4, 0] = -np.inf
    pml[:3, 7, 0] = -np.inf  # empty in the whole first group
    pa = rng.standard_normal((S, rows, D)).astype(np.float32)
    expected = O.merge(pml, pa)
    t_ml, t_a = torch.from_numpy(pml).cuda(), torch.from_numpy(pa).cuda()
    st_ml = torch.empty(2, rows, 2, device="cuda")
    st_a = torch.empty(2, rows, D, device="cuda")
    for gi, sl in enumerate((slice(0, 3), slice(3, 6))):
        capi.merge_to_partial(t_ml[sl].contiguous(), t_a[sl].contiguous(), st_ml[gi], st_a[gi])
    out = torch.empty(rows, D, device="cuda")
    capi.merge_partials(st_ml, st_a, out)
    torch.cuda.synchronize()
    assert U.max_abs(out.cpu().numpy(), expected) < 1e-5
    assert np.isneginf(st_ml[0, 7, 0].item()) and st_ml[0, 7, 1].item() == 0.0
