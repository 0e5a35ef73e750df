"""The context split's exchange over peer memory (bc_merge_exchange) on real
GPUs: two processes, one GPU each, exchange buffers mapped through CUDA IPC.
Every step's result on every rank equals the oracle's unsplit decode of the
whole context; consecutive steps alternate the buffers' parity halves; and a
rank that skips a step (it stays alive and launches nothing) makes the other
rank's device-side wait give up at its limit with BC_ERR_TIMEOUT instead of
hanging. Needs two GPUs of one box (skipped otherwise); no NCCL: the handles
travel through a gloo group."""
import json
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

STEPS = 4
TOL = 1e-4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for sub in ("tests", "oracle", "branchcraft-cuda_b200"):
        sys.path.insert(0, os.path.join(root, sub))
    import torch.distributed as dist

    import bc_capi as C
    import bc_testutil as U
    import oracle as O
    from bc_dist import CollectiveFailed, PeerExchange, p2p_split_kv_decode, shard_pages

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    res = {"errors": [], "timeout": None}
    try:
        rng = np.random.default_rng(77)
        lens = [6000]
        f = U.paged_fixture(rng, 1, 32, 8, 128, lens)
        B, hq, hkv, dim, npg, P = f["shape"]
        shard = shard_pages(npg, world, rank)
        pages = np.ascontiguousarray(f["pages"][:, shard.start:shard.stop])
        length = np.clip(f["lengths"] - shard.start * 16, 0, len(shard) * 16).astype(np.int32)
        s = C.make_shape(B, hq, hkv, dim, pages.shape[1], P)
        k, v = U.to_dev(f["k"]), U.to_dev(f["v"])
        pg, ln = U.to_dev(pages), U.to_dev(length)
        ex = PeerExchange(B * hq, dim)
        C.last_device_error(reset=True)
        for step in range(STEPS):
            q = U.rand_half(np.random.default_rng(1000 + step), (B, hq, dim))
            out = p2p_split_kv_decode(s, U.to_dev(q), k, v, pg, ln, ex, splits=16 if step % 2 else 37)
            torch.cuda.synchronize()
            expected = O.decode(f["shape"], q, f["k"], f["v"], f["pages"], f["lengths"])
            res["errors"].append(float(np.abs(out.cpu().numpy() - expected).max()))
        res["device_error"] = ex.check()
        dist.barrier()
        # rank 1 skips the next step: rank 0's wait gives up at its limit
        if rank == 0:
            q = U.rand_half(np.random.default_rng(9), (B, hq, dim))
            try:
                p2p_split_kv_decode(s, U.to_dev(q), k, v, pg, ln, ex)
                ex.check()
                res["timeout"] = "no error"
            except CollectiveFailed as e:
                res["timeout"] = str(e)
        dist.barrier()
        ex.close()
    finally:
        with open(os.path.join(outdir, f"rank{rank}.json"), "w") as fh:
            json.dump(res, fh)
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_peer_exchange_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs of one box")
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    res = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(world)]
    for r in res:
        assert len(r["errors"]) == STEPS and max(r["errors"]) < TOL, r
        assert r["device_error"] == 0, r
    assert res[0]["timeout"] is not None and "did not arrive" in res[0]["timeout"], res[0]
