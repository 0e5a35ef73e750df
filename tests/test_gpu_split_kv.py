"""One context split across GPUs (BASELINE config 5b), emulated on one GPU.

Each emulated rank owns a contiguous shard of the request's pages and runs
bc_paged_decode_partial on it into one partial buffer; the buffers are stacked
(the all-gather) and bc_merge_gathered reduces them. The result must equal the oracle's unsplit
decode of the whole context. Every rank's kernel runs to completion on its
own; there is no inter-kernel wait, so emulating the ranks as successive
launches is exact. The NCCL exchange itself is covered on CPU ranks (gloo) in
test_dist_cpu.py and on real GPUs by bench.py --workload longctx.
"""
import numpy as np
import pytest
import torch

import bc_testutil as U
import oracle as O
from bc_dist import block_floats, block_views, shard_pages, split_kv_decode

pytestmark = pytest.mark.gpu

TOL = 1e-4  # max-abs on FP32 outputs of N(0,1) inputs, as the decode tests


def _shard_inputs(f, world, rank):
    """This rank's page table and length for request-batch fixture `f`."""
    pages = f["pages"]
    lens = f["lengths"]
    npg = pages.shape[1]
    shard = shard_pages(npg, world, rank)
    mine = np.full((pages.shape[0], max(1, len(shard))), 0, np.int32)
    mine[:, :len(shard)] = pages[:, shard.start:shard.stop]
    my_len = np.clip(lens - shard.start * 16, 0, len(shard) * 16).astype(np.int32)
    return mine, my_len


@pytest.mark.parametrize("world,splits", [(1, 0), (2, 0), (4, 4), (3, 16), (8, 64)])
def test_split_context_matches_unsplit_oracle(world, splits):
    import bc_capi as C

    rng = np.random.default_rng(500 + world * 7 + splits)
    lens = [9000, 4321]  # ragged: request 1 ends inside a shard, later shards empty for it
    f = U.paged_fixture(rng, 2, 32, 8, 128, lens)
    expected = O.decode(f["shape"], f["q"], f["k"], f["v"], f["pages"], f["lengths"])
    q, k, v = U.to_dev(f["q"]), U.to_dev(f["k"]), U.to_dev(f["v"])
    B, hq, _, dim, _, P = f["shape"]
    rows = B * hq
    S = splits if splits > 8 else 1
    blocks = []
    for r in range(world):
        pages, length = _shard_inputs(f, world, r)
        s = C.make_shape(B, hq, 8, dim, pages.shape[1], P)
        buf = torch.full((block_floats(S, rows, dim),), float("nan"), device="cuda")
        pml, pa = block_views(buf, S, rows, dim)
        C.paged_decode_partial(s, q, k, v, U.to_dev(pages), U.to_dev(length), pml, pa, splits)
        blocks.append(buf)

    def merge(g):
        out = torch.empty(rows, dim, device="cuda")
        C.merge_gathered(g, world, S, rows, dim, out)
        return out

    out = split_kv_decode(lambda: blocks[0], merge, lambda t: torch.stack(blocks), S, rows,
                          dim, world)
    torch.cuda.synchronize()
    got = out.view(B, hq, dim).cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - expected).max() <= TOL
    assert C.last_device_error() == 0


def test_partial_rejects_too_many_splits():
    import bc_capi as C

    rng = np.random.default_rng(3)
    f = U.paged_fixture(rng, 1, 32, 8, 128, [64])
    s = C.make_shape(*f["shape"])
    t = [U.to_dev(f[n]) for n in ("q", "k", "v", "pages", "lengths")]
    pml = torch.empty(128, 32, 2, device="cuda")
    pa = torch.empty(128, 32, 128, device="cuda")
    with pytest.raises(C.BranchcraftError):
        C.paged_decode_partial(s, *t, pml, pa, C.MAX_SPLITS + 1)
