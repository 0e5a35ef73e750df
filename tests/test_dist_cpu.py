"""The multi-GPU host logic on CPU ranks (gloo, world size 2): request
sharding covers every request once, and the split-KV exchange protocol of
bc_dist (per-rank FP32 (m, l, acc) partials in one buffer -> one all-gather ->
merge) gives the unsplit decode. The partials here come from a numpy
restatement; on GPUs the same protocol runs with the CUDA entry points and
NCCL. The peer-memory exchange's host logic (PeerExchange: handle exchange,
mapping, epochs, teardown) runs here against a recorded C layer; its kernel
is tested on two GPUs in test_gpu_p2p_exchange.py. The failure tests are in
test_dist_failure_cpu.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bc_dist import block_floats, block_views, shard_pages, shard_requests, split_kv_decode


def test_shard_requests_partition():
    for batch in (1, 7, 8, 1024):
        for world in (1, 2, 4, 8):
            seen = []
            for r in range(world):
                seen += list(shard_requests(batch, world, r))
            assert seen == list(range(batch))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _partial_numpy(q, k, v, pages, length, dim):
    """(m, l, acc) of one request over its shard; m in natural-log units."""
    hq, hkv = q.shape[0], k.shape[2]
    g = hq // hkv
    pml = np.zeros((hq, 2), np.float32)
    pa = np.zeros((hq, dim), np.float32)
    for h in range(hq):
        toks = [k[pages[t // 16], t % 16, h // g] for t in range(length)]
        vals = [v[pages[t // 16], t % 16, h // g] for t in range(length)]
        if not toks:
            pml[h] = (-np.inf, 0.0)
            continue
        s = np.stack(toks) @ q[h] / np.sqrt(dim)
        m = s.max()
        p = np.exp(s - m)
        pml[h] = (m, p.sum())
        pa[h] = p @ np.stack(vals)
    return pml, pa


def _merge_numpy(g_ml, g_a):
    m = g_ml[..., 0].max(axis=0)
    w = np.where(np.isfinite(g_ml[..., 0]), np.exp(g_ml[..., 0] - m), 0.0)
    den = (w * g_ml[..., 1]).sum(axis=0)
    return (w[..., None] * g_a).sum(axis=0) / den[:, None]


def _worker(rank, world, port, data, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, pages, length, dim, per_rank = data
        hq = q.shape[0]
        shard = shard_pages(len(pages), world, rank)
        my_pages = pages[shard.start:shard.stop]

        def local():
            # `per_rank` partials per row: this rank's pages split again, as a
            # GPU keeping its on-chip splits unmerged does, in one buffer.
            buf = torch.zeros(block_floats(per_rank, hq, dim))
            pml, pa = block_views(buf, per_rank, hq, dim)
            for i in range(per_rank):
                sub = shard_pages(len(my_pages), per_rank, i)
                start = shard.start + sub.start
                n = max(0, min(length - start * 16, len(sub) * 16))
                ml, a = _partial_numpy(q, k, v, my_pages[sub.start:sub.stop], n, dim)
                pml[i] = torch.from_numpy(ml)
                pa[i] = torch.from_numpy(a)
            return buf

        def gather(t):
            out = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(out, t)
            return torch.stack(out)

        def merge(g):
            mls, accs = zip(*[block_views(g[r], per_rank, hq, dim) for r in range(world)])
            g_ml = torch.cat(mls).numpy()
            g_a = torch.cat(accs).numpy()
            return torch.from_numpy(_merge_numpy(g_ml, g_a).astype(np.float32))

        out = split_kv_decode(local, merge, gather, per_rank, hq, dim, world)
        result[rank] = out.numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
@pytest.mark.parametrize("per_rank", [1, 2])
def test_split_kv_exchange_gloo_world2(per_rank):
    rng = np.random.default_rng(0)
    hq, hkv, dim, length = 8, 2, 64, 300
    npages = (length + 15) // 16
    k = rng.standard_normal((npages + 3, 16, hkv, dim)).astype(np.float32)
    v = rng.standard_normal((npages + 3, 16, hkv, dim)).astype(np.float32)
    q = rng.standard_normal((hq, dim)).astype(np.float32)
    pages = rng.permutation(npages + 3)[:npages]
    full_ml, full_a = _partial_numpy(q, k, v, pages, length, dim)
    expected = full_a / full_ml[:, 1:2]
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, (q, k, v, pages, length, dim, per_rank),
                                                     result))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(100)
        assert p.exitcode == 0
    for r in range(2):
        assert np.abs(result[r] - expected).max() < 1e-4


class _FakeExchangeC:
    """The bc_capi calls PeerExchange makes, recorded (no GPU): buffers are
    numbered 100 + rank, a mapped peer buffer 200 + the peer's rank."""

    def __init__(self, rank):
        self.rank = rank
        self.calls = []

    def exchange_create(self, world, rows, dim):
        self.calls.append(("create", world, rows, dim))
        return 100 + self.rank, bytes([self.rank]) * 64

    def exchange_open(self, handle):
        self.calls.append(("open", handle[0]))
        return 200 + handle[0]

    def merge_exchange(self, world, rank, epoch, pml, pa, peers, out, stream=None):
        self.calls.append(("merge", world, rank, epoch, peers.tolist()))

    def last_device_error(self, reset=True):
        return 0

    def exchange_close(self, ptr):
        self.calls.append(("close", ptr))

    def exchange_destroy(self, ptr):
        self.calls.append(("destroy", ptr))


def _peer_worker(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from bc_dist import PeerExchange

        C = _FakeExchangeC(rank)
        ex = PeerExchange(32, 128, capi=C, device="cpu")
        for _ in range(3):
            ex.merge(None, None, None)
        ex.check()
        ex.close()
        result[rank] = C.calls
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_peer_exchange_host_logic_gloo_world2():
    """PeerExchange on CPU ranks with a recorded C layer: every rank maps every
    other rank's buffer (never its own), passes the world's buffers in rank
    order, counts the epoch up from 1, and unmaps before it frees its own."""
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(100)
        assert p.exitcode == 0
    for r in range(2):
        calls = result[r]
        other = 1 - r
        assert calls[0] == ("create", 2, 32, 128)
        assert calls[1] == ("open", other)
        peers = [100 + r if w == r else 200 + w for w in range(2)]
        assert calls[2:5] == [("merge", 2, r, e, peers) for e in (1, 2, 3)]
        assert calls[5:] == [("close", 200 + other), ("destroy", 100 + r)]
