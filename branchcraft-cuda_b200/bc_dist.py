"""One ultra-long context split across GPUs (BASELINE config 5b).

Every rank holds a contiguous shard of the request's pages (its own page pool
and page table) and reduces it to one partial softmax state per (request,
q-head): (m, l) and the unnormalised accumulator, in FP32. The partials are
all-gathered over NCCL (16,640 bytes per rank for Hq=32, D=128) and merged on
the device with the same math as the reference merge_kernel
(src/paged_gqa.cu:76-106). Requests that fit on one GPU are instead sharded
by request with no collective at all (`shard_requests`).

The compute steps are parameters so the exchange protocol can be exercised on
CPU ranks (gloo) with a numpy stand-in; the production path passes the CUDA
entry points of bc_capi.
"""
from __future__ import annotations


def shard_requests(batch: int, world: int, rank: int) -> range:
    """Contiguous request range of `rank` (request-sharded configs)."""
    per, extra = divmod(batch, world)
    start = rank * per + min(rank, extra)
    return range(start, start + per + (1 if rank < extra else 0))


def shard_pages(num_pages: int, world: int, rank: int) -> range:
    """Contiguous page range of `rank` for a context split across ranks."""
    return shard_requests(num_pages, world, rank)


def split_kv_decode(local_partial, merge, all_gather, rows: int, dim: int, world: int):
    """Run one distributed decode step.

    local_partial() -> (partial_ml [S, rows, 2], partial_a [S, rows, dim]) of
                       this rank, S >= 1 partials per row (a 2-D pair means S = 1)
    all_gather(t)   -> tensor [world, *t.shape] gathered from every rank
    merge(pml [world*S, rows, 2], pa [world*S, rows, dim]) -> out [rows, dim]
    """
    pml, pa = local_partial()
    if pml.dim() == 2:
        pml, pa = pml.unsqueeze(0), pa.unsqueeze(0)
    S = pml.shape[0]
    assert tuple(pml.shape) == (S, rows, 2) and tuple(pa.shape) == (S, rows, dim)
    g_ml = all_gather(pml)
    g_a = all_gather(pa)
    assert tuple(g_ml.shape) == (world, S, rows, 2)
    return merge(g_ml.reshape(world * S, rows, 2), g_a.reshape(world * S, rows, dim))


def cuda_split_kv_decode(shape, q, k, v, pages, lengths, group, splits: int = 0):
    """Production path: bc_paged_decode_partial on this rank's shard, NCCL
    all_gather_into_tensor, bc_merge_partials. `shape`, `pages`, `lengths`
    describe this rank's shard; returns FP32 [B, Hq, D] on every rank.
    `splits` > 8 keeps that many unmerged partials per row on every rank (all
    of them are gathered and merged at once); otherwise each rank sends one."""
    import torch
    import torch.distributed as dist

    import bc_capi as C

    world = dist.get_world_size(group)
    rows = shape.batch * shape.query_heads
    dev = q.device
    S = splits if splits > 8 else 1

    def local_partial():
        pml = torch.empty(S, rows, 2, device=dev, dtype=torch.float32)
        pa = torch.empty(S, rows, shape.dim, device=dev, dtype=torch.float32)
        C.paged_decode_partial(shape, q, k, v, pages, lengths, pml, pa, splits)
        return pml, pa

    def all_gather(t):
        out = torch.empty((world,) + tuple(t.shape), device=dev, dtype=t.dtype)
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
        return out

    def merge(g_ml, g_a):
        out = torch.empty(rows, shape.dim, device=dev, dtype=torch.float32)
        C.merge_partials(g_ml, g_a, out)
        return out

    out = split_kv_decode(local_partial, merge, all_gather, rows, shape.dim, world)
    return out.view(shape.batch, shape.query_heads, shape.dim)
