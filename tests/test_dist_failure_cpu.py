"""Failure handling of the split-KV exchange on CPU ranks (gloo, world size 2),
with the failure made on the host: a rank that leaves between steps, and a
rank that passes the step gate but never posts its collective (a dropped
message). The survivor must return an error within its deadline instead of
waiting for the peer (bc_dist.StepGate, bc_dist.wait_collective)."""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bc_dist import CollectiveFailed, PeerLost, StepGate, wait_collective


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _exchange(step, gate, deadline):
    gate.enter(step)
    t = torch.full((4,), float(dist.get_rank() + step))
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    work = dist.all_gather(out, t, async_op=True)
    wait_collective(work, deadline_s=deadline)
    return [float(x[0]) for x in out]


def _worker(rank, world, port, scenario, leaver, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    store = dist.distributed_c10d._get_default_store()
    gate = StepGate(store, rank, world, timeout_s=2.0)
    # step 0: everyone takes part
    result[f"step0/{rank}"] = _exchange(0, gate, deadline=10.0)
    if rank == leaver:
        if scenario == "drop":
            # passes the gate of step 1, then never posts its collective
            gate.enter(1)
            time.sleep(6.0)
        os._exit(0)  # leaves between steps: nothing of it is in flight
    t0 = time.monotonic()
    try:
        _exchange(1, gate, deadline=1.5)
        result[f"outcome/{rank}"] = "completed"
    except PeerLost:
        result[f"outcome/{rank}"] = "PeerLost"
    except CollectiveFailed:
        result[f"outcome/{rank}"] = "CollectiveFailed"
    result[f"elapsed/{rank}"] = time.monotonic() - t0
    os._exit(0)  # the peer is gone: do not wait for it in the group's teardown


def _run(scenario, leaver):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, scenario, leaver, result))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return dict(result)


@pytest.mark.timeout(120)
@pytest.mark.parametrize("leaver", [1, 0])
def test_rank_leaving_between_steps_is_found_at_the_gate(leaver):
    """The leaving rank exits after step 0; the survivor's gate for step 1
    raises PeerLost within about its 2 s timeout (leaver 0 also takes the
    store's host process with it)."""
    r = _run("leave", leaver)
    survivor = 1 - leaver
    assert r[f"step0/{survivor}"] == [0.0, 1.0]
    assert r[f"outcome/{survivor}"] == "PeerLost"
    assert r[f"elapsed/{survivor}"] < 10.0


@pytest.mark.timeout(120)
def test_dropped_collective_misses_its_deadline():
    """Rank 1 passes the gate of step 1 but never posts its all-gather: rank
    0's collective is abandoned at its 1.5 s host deadline."""
    r = _run("drop", 1)
    assert r["step0/0"] == [0.0, 1.0]
    assert r["outcome/0"] == "CollectiveFailed"
    assert r["elapsed/0"] < 10.0
