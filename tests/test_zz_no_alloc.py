"""bc_decode_static_scratch — the decode entry point for callers that cannot
allocate device memory (a plugin handed only its inputs and outputs, or a decode
loop whose memory plan forbids per-step allocation): its split partials live in
a fixed array inside the library instead of caller scratch.

Checked through the C ABI against the existing entry point (bc_decode with
caller scratch) and against the CPU oracle, within the tolerance the decode
tests use, on calls in a row with different inputs and split counts, so stale
contents of the shared array from one call cannot leak into the next. The
split counts cover every path the entry point has: 64 and 16 (the global merge
that bc_decode also takes), 4 (here forced through the array and the global
merge, where bc_decode merges on chip) and 1 (no merge, the array unused).
This file is collected last on purpose; it also passes alone in a fresh
process (the first call on the device performs the array's address look-up).
"""
import ctypes

import numpy as np
import pytest
import torch

import bc_testutil as U
import oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-4  # max-abs, as in tests/test_gpu_decode.py


def _inputs(seed, batch, ctx):
    rng = np.random.default_rng(seed)
    lens = [ctx - (i % 3) * ctx // 5 for i in range(batch)]
    lens[-1] = 0  # an empty sequence: zeros from both paths
    f = U.paged_fixture(rng, batch, 32, 8, 128, lens)
    return f, [U.to_dev(f[n]) for n in ("q", "k", "v", "pages", "lengths")]


def _reference_call(C, f, t, splits):
    s = C.make_shape(*f["shape"])
    rows = s.batch * s.query_heads
    out = torch.full((s.batch, s.query_heads, s.dim), float("nan"), device="cuda")
    pa = torch.empty(splits * rows * s.dim, device="cuda")
    pml = torch.empty(splits * rows * 2, device="cuda")
    C.decode(s, *t, out, pa, pml, splits)
    return out


def test_static_scratch_matches_caller_scratch_on_two_calls():
    import bc_capi as C

    # (seed, batch, context, splits): consecutive calls share the array
    calls = [(101, 4, 6000, 64), (202, 3, 2500, 16), (303, 2, 3100, 4), (404, 3, 900, 1)]
    runs = []
    for seed, batch, ctx, splits in calls:
        f, t = _inputs(seed, batch, ctx)
        out = torch.full((batch, 32, 128), float("nan"), device="cuda")
        C.decode_static_scratch(C.make_shape(*f["shape"]), *t, out, splits)
        runs.append((f, t, splits, out))
    torch.cuda.synchronize()
    for f, t, splits, out in runs:
        ref = _reference_call(C, f, t, splits)
        torch.cuda.synchronize()
        expected = O.decode(f["shape"], f["q"], f["k"], f["v"], f["pages"], f["lengths"])
        assert torch.isfinite(out).all()
        assert (out - ref).abs().max().item() <= TOL, f"splits={splits} vs bc_decode"
        assert U.max_abs(out.cpu().numpy(), expected) <= TOL, f"splits={splits} vs oracle"
    assert C.last_device_error() == 0


def test_static_scratch_rejects_oversize_without_launching():
    import bc_capi as C

    f, t = _inputs(7, 4, 300)
    s = C.make_shape(*f["shape"])
    out = torch.zeros(4, 32, 128, device="cuda")
    # 64 splits x 4 x 32 rows x (128 + 2) fits; 64 x 8 x 32 x 130 does not.
    big = C.make_shape(8, 32, 8, 128, s.max_pages, s.physical_pages)
    rc = C.lib().bc_decode_static_scratch(ctypes.byref(big), *[C._ptr(x) for x in t],
                                          C._ptr(out), 64, C._stream())
    assert rc == 1  # cudaErrorInvalidValue
    assert out.abs().max().item() == 0.0
