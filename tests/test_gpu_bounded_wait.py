"""The bounded waits of the kernels, exercised on the GPU without a fault: a
self-test launch whose CTAs wait on a barrier that nothing completes. Each
wait gives up after a short limit and sets BC_ERR_TIMEOUT; the first one to
give up aborts the launch, so CTAs of later waves return at once and the
launch costs about one limit instead of one per wave. A later launch carries
a new abort token and runs normally."""
import numpy as np
import pytest
import torch

import bc_testutil as U
import oracle as O

pytestmark = pytest.mark.gpu


def test_stalled_launch_gives_up_after_one_limit():
    import bc_capi as C

    limit_us = 20000
    ctas = 148 * 6  # 180 KB of shared memory each: one CTA per SM, six waves
    C.last_device_error()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    C.selftest_bounded_wait(ctas, 180 * 1024, limit_us)
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b)
    assert C.last_device_error() & C.ERR_TIMEOUT
    assert 0.8 * limit_us / 1000 <= ms < 3 * limit_us / 1000, ms  # not 6 limits

    # the next launch has its own token: a decode with waits in its pipeline
    rng = np.random.default_rng(4)
    f = U.paged_fixture(rng, 2, 32, 8, 128, [3000, 1700])
    s = C.make_shape(*f["shape"])
    out = torch.empty(2, 32, 128, device="cuda")
    C.paged_decode(s, *[U.to_dev(f[n]) for n in ("q", "k", "v", "pages", "lengths")], out, 0)
    torch.cuda.synchronize()
    assert C.last_device_error() == 0
    expected = O.decode(f["shape"], f["q"], f["k"], f["v"], f["pages"], f["lengths"])
    assert U.max_abs(out.cpu().numpy(), expected) < 1e-4


def test_selftest_rejects_bad_arguments():
    import bc_capi as C

    with pytest.raises(C.BranchcraftError):
        C.selftest_bounded_wait(0, 0, 1000)
    with pytest.raises(C.BranchcraftError):
        C.selftest_bounded_wait(4, 0, 5000000)
