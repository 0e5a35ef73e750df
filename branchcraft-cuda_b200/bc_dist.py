"""One ultra-long context split across GPUs (BASELINE config 5b), and the
host-side failure handling of that exchange.

Every rank holds a contiguous shard of the request's pages (its own page pool
and page table) and reduces it to partial softmax states per (request,
q-head): (m, l) and the unnormalised accumulator, in FP32. A rank's partials
sit in ONE buffer — its `splits * rows` (m, l) pairs, then its
`splits * rows * dim` accumulators — so a single NCCL all-gather of that
buffer (one partial per row: 16,640 bytes per rank for Hq=32, D=128; a rank
first reduces its own on-device splits with bc_merge_to_partial) brings every rank's
partials to every rank, where one merge launch (bc_merge_gathered, the math of
the reference merge_kernel, src/paged_gqa.cu:76-106) reduces them. Requests
that fit on one GPU are instead sharded by request with no collective at all
(`shard_requests`).

Failure handling (the reference has no distributed code; these are the rules
of a multi-GPU deployment of it):
  * `StepGate`: before a step's collective every rank posts its step number
    to the process group's key-value store and waits, for a bounded time, for
    every peer's post of the same step. A rank that left between steps is
    found on the host before anyone launches the collective (`PeerLost`).
  * `wait_collective`: an issued collective is polled under a host deadline;
    the communicator's asynchronous error (ncclCommGetAsyncError, through
    `ProcessGroupNCCL.get_error`) is checked on every poll, and on an error or
    at the deadline the communicator is aborted (ncclCommAbort, through
    `ProcessGroupNCCL.abort`) and `CollectiveFailed` raised, so no rank waits
    forever on a peer that never joined.
  * `exchange_group`: the NCCL communicator of the exchange is created
    non-blocking (NCCL config `blocking = 0`), so an abort never waits behind
    a collective that cannot finish.

The compute steps are parameters so the exchange protocol can be exercised on
CPU ranks (gloo) with a numpy stand-in; the production path passes the CUDA
entry points of bc_capi.

`PeerExchange` + `p2p_split_kv_decode` replace the all-gather with peer
memory: one kernel per rank (bc_merge_exchange) reduces the rank's splits,
writes the reduced state into every rank's exchange buffer over NVLink
(CUDA IPC mappings made once), waits for the peers' flags on the device
(bounded: BC_ERR_TIMEOUT, checked by `PeerExchange.check`) and merges the
world's states — no collective library call on the data path. The handles
are exchanged once through the process group (any backend).
"""
from __future__ import annotations

import datetime
import time


class PeerLost(RuntimeError):
    """A peer did not reach the step gate in time (it left between steps)."""


class CollectiveFailed(RuntimeError):
    """A collective reported an asynchronous error or missed its deadline."""


def shard_requests(batch: int, world: int, rank: int) -> range:
    """Contiguous request range of `rank` (request-sharded configs)."""
    per, extra = divmod(batch, world)
    start = rank * per + min(rank, extra)
    return range(start, start + per + (1 if rank < extra else 0))


def shard_pages(num_pages: int, world: int, rank: int) -> range:
    """Contiguous page range of `rank` for a context split across ranks."""
    return shard_requests(num_pages, world, rank)


def block_floats(splits: int, rows: int, dim: int) -> int:
    """Floats in one rank's partial buffer: (m, l) pairs, then accumulators."""
    return splits * rows * (2 + dim)


def block_views(buf, splits: int, rows: int, dim: int):
    """(partial_ml [S, rows, 2], partial_a [S, rows, dim]) views of a flat
    per-rank partial buffer."""
    n_ml = splits * rows * 2
    return (buf[:n_ml].view(splits, rows, 2),
            buf[n_ml:n_ml + splits * rows * dim].view(splits, rows, dim))


def split_kv_decode(local_partial, merge, all_gather, splits: int, rows: int, dim: int,
                    world: int):
    """Run one distributed decode step.

    local_partial() -> flat buffer of this rank's `splits` partials per row
                       (block_floats(splits, rows, dim) floats, `block_views`)
    all_gather(t)   -> [world, t.numel()] gathered from every rank
    merge(g)        -> out [rows, dim] from the gathered [world, n] buffer
    """
    buf = local_partial()
    assert buf.dim() == 1 and buf.numel() == block_floats(splits, rows, dim), tuple(buf.shape)
    g = all_gather(buf)
    assert tuple(g.shape) == (world, buf.numel()), tuple(g.shape)
    return merge(g)


# ------------------------------------------------------------ failure handling
class StepGate:
    """Host-side liveness check between steps through the store every rank of
    a process group shares. `enter(step)` posts this rank's arrival at `step`
    and returns once every peer has posted the same step, or raises
    `PeerLost` after `timeout_s`. A rank leaves only between steps (none of
    its kernels or collectives in flight), so the survivors learn of it here,
    before they launch the step's collective."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 2.0,
                 prefix: str = "bc_gate"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout = datetime.timedelta(seconds=timeout_s)
        self.prefix = prefix

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def enter(self, step: int) -> None:
        peers = [self._key(step, r) for r in range(self.world) if r != self.rank]
        try:
            self.store.set(self._key(step, self.rank), "1")
            if peers:
                self.store.wait(peers, self.timeout)
        except Exception as e:  # a timeout, or the store's host is gone
            raise PeerLost(f"step {step}: not every peer arrived within "
                           f"{self.timeout.total_seconds():.1f} s ({e})") from e


def wait_collective(work, group=None, deadline_s: float = 5.0, poll_s: float = 2e-4):
    """Poll an async collective's work handle under a host deadline. On the
    communicator's asynchronous error, or when the deadline passes, abort the
    communicator (if the backend can) and raise `CollectiveFailed`."""
    t0 = time.monotonic()
    backend = _nccl_backend(group)
    while not work.is_completed():
        err = _async_error(backend)
        if err:
            _abort(backend)
            raise CollectiveFailed(f"communicator reported asynchronous error {err}")
        if time.monotonic() - t0 > deadline_s:
            _abort(backend)
            raise CollectiveFailed(f"collective did not complete within {deadline_s:.1f} s")
        time.sleep(poll_s)
    err = _async_error(backend)
    if err:
        _abort(backend)
        raise CollectiveFailed(f"communicator reported asynchronous error {err}")


def _nccl_backend(group):
    """The ProcessGroupNCCL behind `group` (None when not NCCL)."""
    try:
        import torch
        import torch.distributed as dist

        pg = group if group is not None else dist.distributed_c10d._get_default_group()
        be = pg._get_backend(torch.device("cuda"))
        return be if hasattr(be, "get_error") else None
    except Exception:
        return None


def _async_error(backend) -> int:
    if backend is None:
        return 0
    try:
        return int(backend.get_error())
    except Exception:
        return 0


def _abort(backend) -> None:
    if backend is None:
        return
    try:
        backend.abort()
    except Exception:
        pass


def exchange_group(ranks=None, timeout_s: float = 30.0):
    """A process group for the split-KV exchange whose NCCL communicator is
    non-blocking (NCCL config `blocking = 0`) with a short timeout; falls back
    to a default-options group on backends without NCCL options."""
    import torch.distributed as dist

    timeout = datetime.timedelta(seconds=timeout_s)
    try:
        from torch.distributed import ProcessGroupNCCL

        opts = ProcessGroupNCCL.Options()
        opts.config.blocking = 0
        opts._timeout = timeout  # (the same value as the kwarg, which wins)
        return dist.new_group(ranks=ranks, timeout=timeout, backend="nccl", pg_options=opts)
    except Exception:
        return dist.new_group(ranks=ranks, timeout=timeout)


# ------------------------------------------------------------ production path
def cuda_split_kv_decode(shape, q, k, v, pages, lengths, group=None, splits: int = 0,
                         deadline_s: float = 0.0, gate: StepGate = None, step: int = 0):
    """Production path: bc_paged_decode_partial on this rank's shard into one
    partial buffer, one NCCL all_gather_into_tensor of it, bc_merge_gathered.
    `shape`, `pages`, `lengths` describe this rank's shard; returns FP32
    [B, Hq, D] on every rank. `splits` > 8 runs that many splits on the rank
    (global partials, reduced on the rank by bc_merge_to_partial); every rank
    sends one partial per row either way. With `gate`, every rank passes the step gate first; with
    `deadline_s` > 0 the collective is waited for under that host deadline
    (the host then synchronises with the step)."""
    import torch
    import torch.distributed as dist

    import bc_capi as C

    world = dist.get_world_size(group)
    rows = shape.batch * shape.query_heads
    dev = q.device
    S = splits if splits > 8 else 1
    if gate is not None:
        gate.enter(step)

    def local_partial():
        part = torch.empty(block_floats(S, rows, shape.dim), device=dev, dtype=torch.float32)
        pml, pa = block_views(part, S, rows, shape.dim)
        C.paged_decode_partial(shape, q, k, v, pages, lengths, pml, pa, splits)
        if S == 1:
            return part
        # the rank's splits reduced to ONE partial per row before the exchange
        buf = torch.empty(block_floats(1, rows, shape.dim), device=dev, dtype=torch.float32)
        ml1, a1 = block_views(buf, 1, rows, shape.dim)
        C.merge_to_partial(pml, pa, ml1[0], a1[0])
        return buf

    def all_gather(t):
        out = torch.empty((world, t.numel()), device=dev, dtype=t.dtype)
        work = dist.all_gather_into_tensor(out, t, group=group, async_op=deadline_s > 0)
        if deadline_s > 0:
            wait_collective(work, group, deadline_s)
        return out

    def merge(g):
        out = torch.empty(rows, shape.dim, device=dev, dtype=torch.float32)
        C.merge_gathered(g, world, 1, rows, shape.dim, out)
        return out

    out = split_kv_decode(local_partial, merge, all_gather, 1, rows, shape.dim, world)
    return out.view(shape.batch, shape.query_heads, shape.dim)


class PeerExchange:
    """The peer-memory exchange of one context split: this rank's exchange
    buffer, the peers' buffers mapped through CUDA IPC, and the device array
    of their addresses in rank order. One per (group, rows, dim); `merge`
    runs one step (every rank calls it the same number of times); `close`
    unmaps and frees after every rank's last step."""

    def __init__(self, rows: int, dim: int, group=None, capi=None, device=None):
        import torch
        import torch.distributed as dist

        self.C = capi if capi is not None else __import__("bc_capi")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows, self.dim = rows, dim
        self.own, handle = self.C.exchange_create(self.world, rows, dim)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.mapped = []
        ptrs = []
        for w, h in enumerate(handles):
            if w == self.rank:
                ptrs.append(self.own)
            else:
                p = self.C.exchange_open(h)
                self.mapped.append(p)
                ptrs.append(p)
        self.peers = torch.tensor(ptrs, dtype=torch.int64,
                                  device=device if device is not None else torch.cuda.current_device())
        self.epoch = 0

    def merge(self, partial_ml, partial_a, out, stream=None):
        """One step: this rank's [S, rows, 2] / [S, rows, dim] partials in, the
        merge of every rank's partials in `out` [rows, dim]."""
        self.epoch += 1
        self.C.merge_exchange(self.world, self.rank, self.epoch, partial_ml, partial_a,
                              self.peers, out, stream)

    def check(self):
        """Raises CollectiveFailed when a device-side wait for a peer gave up
        (synchronises the device). The exchange is not reusable after that (a
        peer may have published an epoch this rank gave up on): close it and
        build a new one."""
        err = self.C.last_device_error(reset=True)
        if err & 8:  # BC_ERR_TIMEOUT
            raise CollectiveFailed(
                f"rank {self.rank}: a peer's partials did not arrive within the wait limit "
                f"(device error word {err:#x})")
        return err

    def close(self):
        """Unmap the peers' buffers, wait for every rank to stop writing into
        this one, free it."""
        import torch
        import torch.distributed as dist

        if self.peers.is_cuda:
            torch.cuda.synchronize()
        for p in self.mapped:
            self.C.exchange_close(p)
        self.mapped = []
        dist.barrier(group=self.group)
        if self.own:
            self.C.exchange_destroy(self.own)
            self.own = 0


def p2p_split_kv_decode(shape, q, k, v, pages, lengths, exchange: PeerExchange,
                        splits: int = 37, gate: StepGate = None, step: int = 0):
    """Production path over peer memory: bc_paged_decode_partial on this
    rank's shard (`splits` > 8: every split keeps its partial), then ONE
    bc_merge_exchange launch (local reduction, the exchange, the merge);
    returns FP32 [B, Hq, D] on every rank."""
    import torch

    C = exchange.C
    rows = shape.batch * shape.query_heads
    if gate is not None:
        gate.enter(step)
    S = splits if splits > 8 else 1  # (up to 8 splits merge in a cluster: one partial)
    part = torch.empty(block_floats(S, rows, shape.dim), device=q.device, dtype=torch.float32)
    pml, pa = block_views(part, S, rows, shape.dim)
    C.paged_decode_partial(shape, q, k, v, pages, lengths, pml, pa, splits)
    out = torch.empty(rows, shape.dim, device=q.device, dtype=torch.float32)
    exchange.merge(pml, pa, out)
    return out.view(shape.batch, shape.query_heads, shape.dim)
