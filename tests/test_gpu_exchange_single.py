"""bc_merge_exchange on ONE GPU, with no kernel waiting on another: the
world's other ranks are emulated by their exchange-buffer contents, written
by the host before rank 0's launch (their states and the flags that publish
them), so rank 0's kernel only reads flags that are already set — or, in the
timeout case, a flag nothing sets. Checks: the merge equals the oracle's
unsplit decode of the whole context; rank 0's own state lands in every
rank's slot for it with its flags; consecutive epochs alternate the parity
halves; an unpublished peer makes the bounded wait give up with
BC_ERR_TIMEOUT and zero rows. The two-process test on two GPUs is
test_gpu_p2p_exchange.py."""
import numpy as np
import pytest
import torch

import bc_testutil as U
import oracle as O
from bc_dist import block_floats, block_views, shard_pages

pytestmark = pytest.mark.gpu

ROWS_PER_BLOCK = 4


class _DeviceView:
    """A raw device allocation seen as a torch tensor (no copy)."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3}


def _buffer_views(ptr, world, rows, dim, nbytes):
    raw = torch.as_tensor(_DeviceView(ptr, nbytes), device="cuda")
    stride = dim + 4
    states_floats = 2 * world * rows * stride
    flags_off = (states_floats * 4 + 255) // 256 * 256
    blocks = (rows + ROWS_PER_BLOCK - 1) // ROWS_PER_BLOCK
    states = raw[:states_floats * 4].view(torch.float32).view(2, world, rows, stride)
    flags = raw[flags_off:flags_off + 2 * world * blocks * 4].view(torch.int32).view(2, world, blocks)
    return states, flags


def _context(world, seed=11, length=5000):
    rng = np.random.default_rng(seed)
    f = U.paged_fixture(rng, 1, 32, 8, 128, [length])
    B, hq, hkv, dim, npg, P = f["shape"]
    k, v = U.to_dev(f["k"]), U.to_dev(f["v"])
    shards = []
    for r in range(world):
        sh = shard_pages(npg, world, r)
        pages = np.ascontiguousarray(f["pages"][:, sh.start:sh.stop])
        ln = np.clip(f["lengths"] - sh.start * 16, 0, len(sh) * 16).astype(np.int32)
        shards.append((pages, ln))
    return f, k, v, shards


def _partials(C, f, k, v, pages, ln, q, splits):
    B, hq, hkv, dim, _, P = f["shape"]
    s = C.make_shape(B, hq, hkv, dim, pages.shape[1], P)
    S = splits if splits > 8 else 1
    buf = torch.empty(block_floats(S, B * hq, dim), device="cuda")
    pml, pa = block_views(buf, S, B * hq, dim)
    C.paged_decode_partial(s, q, k, v, U.to_dev(pages), U.to_dev(ln), pml, pa, splits)
    return pml, pa


@pytest.mark.parametrize("world", [1, 4])
def test_emulated_world_matches_unsplit_oracle(world):
    import bc_capi as C

    f, k, v, shards = _context(world)
    rows, dim = 32, 128
    nbytes = C.exchange_bytes(world, rows, dim)
    bufs = [C.exchange_create(world, rows, dim)[0] for _ in range(world)]
    try:
        views = [_buffer_views(b, world, rows, dim, nbytes) for b in bufs]
        peers = torch.tensor(bufs, dtype=torch.int64, device="cuda")
        C.last_device_error(reset=True)
        for epoch in (1, 2, 3):
            par = epoch & 1
            q_h = U.rand_half(np.random.default_rng(100 + epoch), (1, 32, dim))
            q = U.to_dev(q_h)
            # ranks 1.. publish their reduced states in rank 0's buffer
            states0, flags0 = views[0]
            for w in range(1, world):
                pml, pa = _partials(C, f, k, v, *shards[w], q, 37)
                ml1 = torch.empty(1, rows, 2, device="cuda")
                a1 = torch.empty(1, rows, dim, device="cuda")
                C.merge_to_partial(pml, pa, ml1[0], a1[0])
                states0[par, w, :, 0:2] = ml1[0]
                states0[par, w, :, 4:] = a1[0]
                flags0[par, w, :] = epoch
            torch.cuda.synchronize()
            pml, pa = _partials(C, f, k, v, *shards[0], q, 37 if epoch != 2 else 16)
            out = torch.full((rows, dim), float("nan"), device="cuda")
            C.merge_exchange(world, 0, epoch, pml, pa, peers, out)
            torch.cuda.synchronize()
            expected = O.decode(f["shape"], q_h, f["k"], f["v"], f["pages"], f["lengths"])
            assert U.max_abs(out.cpu().numpy().reshape(expected.shape), expected) < 1e-4, epoch
            # rank 0's state reached every rank's slot for it, with its flags
            for w in range(world):
                st, fl = views[w]
                assert (fl[par, 0] == epoch).all(), (epoch, w)
                assert torch.equal(st[par, 0], views[0][0][par, 0])
        assert C.last_device_error() == 0
    finally:
        for b in bufs:
            C.exchange_destroy(b)


def test_unpublished_peer_times_out():
    """A peer whose flag nothing sets: the wait gives up at its limit, the
    error word says BC_ERR_TIMEOUT, the rows are zero, the device is usable."""
    import bc_capi as C

    f, k, v, shards = _context(2)
    rows, dim = 32, 128
    bufs = [C.exchange_create(2, rows, dim)[0] for _ in range(2)]
    try:
        peers = torch.tensor(bufs, dtype=torch.int64, device="cuda")
        q = U.to_dev(U.rand_half(np.random.default_rng(5), (1, 32, dim)))
        pml, pa = _partials(C, f, k, v, *shards[0], q, 37)
        out = torch.full((rows, dim), float("nan"), device="cuda")
        C.last_device_error(reset=True)
        C.merge_exchange(2, 0, 1, pml, pa, peers, out)
        torch.cuda.synchronize()
        assert C.last_device_error() & 8
        assert torch.count_nonzero(out).item() == 0
        # the context still works
        out2 = torch.empty_like(out)
        C.merge_to_partial(pml, pa, torch.empty(rows, 2, device="cuda"), out2)
        torch.cuda.synchronize()
        assert C.last_device_error() == 0
    finally:
        for b in bufs:
            C.exchange_destroy(b)
