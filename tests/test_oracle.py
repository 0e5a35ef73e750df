"""The CPU oracle pinned against the reference (runs without a GPU).

Golden vectors: tests/golden/reference_cases.npz holds, for every known-answer
case of the reference's `branchcraft test` (src/main.cu:252-262, :318-352), the
SHA-256 of the reference-generated inputs and the reference CPU oracle's
output, produced by tests/golden/make_golden.py from the reference's own code.
"""
import numpy as np
import pytest

import bc_testutil as U
import oracle as O


def test_half_conversion_exhaustive():
    bits = np.arange(65536, dtype=np.uint16)
    got = O.h2f(bits)
    want = bits.view(np.float16).astype(np.float32)
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert same.all()
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200_000).astype(np.float32) * s
                        for s in (1e-7, 1e-5, 1e-3, 1.0, 1e3, 6e4)])
    x = np.concatenate([x, np.array([65504, 65519.99, 65520, 6.1e-5, 5.96e-8, 2.98e-8, 0.0,
                                     -0.0, np.inf, -np.inf], np.float32)])
    with np.errstate(over="ignore"):
        assert np.array_equal(O.f2h(x), x.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("case", range(len(U.DECODE_CASES)))
def test_decode_oracle_matches_reference_golden(case):
    g = U.golden()
    b, hq, hkv, d, lens = U.DECODE_CASES[case]
    f = O.ref_fixture(b, hq, hkv, d, lens, 17)
    assert U.digest(f["q"], f["k"], f["v"], f["pages"]) == str(g[f"decode{case}_sha"])
    out = O.decode(f["shape"], f["q"], f["k"], f["v"], f["pages"], f["lengths"])
    assert np.array_equal(out, g[f"decode{case}_out"])  # bit-exact


@pytest.mark.parametrize("case", range(len(U.TREE_CASES)))
def test_tree_oracle_matches_reference_golden(case):
    g = U.golden()
    prefix, d, seed = U.TREE_CASES[case]
    f = O.ref_tree_fixture(2, prefix, 7, d, seed)
    assert U.digest(f["q"], f["k"], f["v"], f["pages"], f["lengths"], f["draft_q"],
                    f["draft_k"], f["draft_v"], f["parent"]) == str(g[f"tree{case}_sha"])
    out = O.tree(f["shape"], 7, f["draft_q"], f["k"], f["v"], f["pages"], f["lengths"],
                 f["draft_k"], f["draft_v"], f["parent"])
    assert np.array_equal(out, g[f"tree{case}_out"])  # bit-exact


def test_packed_oracle_equals_decode_oracle_on_reference_layout():
    """Interleaving paged K/V as [P, Hkv, 16, 2D] (V at +D) must not change
    the result: the packed oracle equals the decode oracle (then FP16)."""
    f = O.ref_fixture(3, 12, 3, 64, [7, 40, 0], 5)
    P, _, hkv, d = f["k"].shape
    packed = np.concatenate([f["k"], f["v"]], axis=-1).transpose(0, 2, 1, 3).copy()
    bs, hs, ss = hkv * 16 * 2 * d, 16 * 2 * d, 2 * d
    _, f32 = O.packed_decode(f["shape"], f["q"], packed, f["pages"], f["lengths"], bs, hs, ss, d,
                             1 / np.sqrt(d), want_f32=True)
    ref = O.decode(f["shape"], f["q"], f["k"], f["v"], f["pages"], f["lengths"])
    assert np.abs(f32 - ref).max() < 1e-6


def test_merge_oracle_splits_reassemble_decode():
    """Splitting a sequence into chunks, attending each, and merging the
    (m, l, acc) partials reproduces the unsplit result."""
    rng = np.random.default_rng(1)
    d, n = 64, 300
    q = rng.standard_normal(d)
    k = rng.standard_normal((n, d))
    v = rng.standard_normal((n, d))
    s = k @ q / np.sqrt(d)
    full = (np.exp(s - s.max()) @ v) / np.exp(s - s.max()).sum()
    chunks = np.array_split(np.arange(n), 5)
    pml = np.zeros((5, 1, 2), np.float32)
    pa = np.zeros((5, 1, d), np.float32)
    for i, c in enumerate(chunks):
        m = s[c].max()
        pml[i, 0] = (m, np.exp(s[c] - m).sum())
        pa[i, 0] = np.exp(s[c] - m) @ v[c]
    assert np.abs(O.merge(pml, pa)[0] - full).max() < 1e-5


@pytest.mark.skipif(not O.ref_available(), reason="reference-built library not present")
def test_oracle_bitexact_vs_reference_build_on_random_cases():
    rng = np.random.default_rng(9)
    for _ in range(3):
        lens = list(rng.integers(0, 300, size=3))
        a = O.ref_fixture(3, 8, 2, 64, lens, int(rng.integers(1 << 30)))
        ours = O.decode(a["shape"], a["q"], a["k"], a["v"], a["pages"], a["lengths"])
        theirs = O.ref_cpu_reference(a["shape"], a["q"], a["k"], a["v"], a["pages"], a["lengths"])
        assert np.array_equal(ours, theirs)
