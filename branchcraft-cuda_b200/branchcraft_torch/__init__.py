"""PyTorch dispatcher bindings for the B200 branchcraft kernels.

Importing this module loads the native operator library (``_C*.so`` next to
this file, which links ``lib/libbranchcraft.so``) and registers fake (meta)
kernels so ``torch.compile`` and FakeTensor tracing see every op's output.
The public API is ``torch.ops.branchcraft``; the functions below are thin
wrappers with the reference's names (python/branchcraft_torch/__init__.py).
There is no fallback: a missing extension is an ImportError.
"""
from pathlib import Path

import torch

_library = next(Path(__file__).parent.glob("_C*.so"), None)
if _library is None:
    raise ImportError("branchcraft CUDA extension is missing; run "
                      "`python branchcraft-cuda_b200/build.py`")
torch.ops.load_library(str(_library))


@torch.library.register_fake("branchcraft::tree_verify")
def _fake_tree_verify(q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent):
    return q.new_empty(q.shape, dtype=torch.float32)


@torch.library.register_fake("branchcraft::packed_decode_out")
def _fake_packed_decode_out(q, packed_kv, pages, lengths, output, scale):
    return output


@torch.library.register_fake("branchcraft::commit_path_")
def _fake_commit_path(cache_k, cache_v, draft_k, draft_v, path_nodes, dest_pages,
                      dest_slots, request):
    return None


@torch.library.register_fake("branchcraft::paged_decode")
def _fake_paged_decode(q, k, v, pages, lengths, splits=0):
    return q.new_empty(q.shape, dtype=torch.float32)


@torch.library.register_fake("branchcraft::tree_verify_out")
def _fake_tree_verify_out(q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent,
                          output):
    return output


@torch.library.register_fake("branchcraft::packed_decode_kv_out")
def _fake_packed_decode_kv_out(q, k_cache, v_cache, pages, lengths, output, scale, splits=0):
    return output


@torch.library.register_fake("branchcraft::commit_batch_")
def _fake_commit_batch(cache_k, cache_v, draft_k, draft_v, clone_src, clone_dst,
                       entry_request, entry_node, entry_page, entry_slot):
    return None


def tree_verify(q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent):
    """Return FP32 [batch, candidate, query head, dimension] outputs."""
    return torch.ops.branchcraft.tree_verify(
        q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent)


def tree_verify_out(q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent, output):
    """Tree verify into a preallocated FP32 or FP16 output (CUDA-graph safe)."""
    return torch.ops.branchcraft.tree_verify_out(
        q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent, output)


def packed_decode_out(q, packed_kv, pages, lengths, output, scale):
    """Decode into a preallocated FP16 output (safe for CUDA graph capture)."""
    return torch.ops.branchcraft.packed_decode_out(q, packed_kv, pages, lengths, output, scale)


def packed_decode_kv_out(q, k_cache, v_cache, pages, lengths, output, scale, splits=0):
    """Decode from separate K / V views [P, Hkv, 16, D] of one cache (e.g. vLLM's
    [num_blocks, 2, 16, Hkv, D] as cache[:, 0].transpose(1, 2) and cache[:, 1]...)."""
    return torch.ops.branchcraft.packed_decode_kv_out(
        q, k_cache, v_cache, pages, lengths, output, scale, splits)


def paged_decode(q, k, v, pages, lengths, splits=0):
    """Paged GQA decode, FP32 [batch, query heads, dim]; splits 0 = automatic."""
    return torch.ops.branchcraft.paged_decode(q, k, v, pages, lengths, splits)


def commit_path_(cache_k, cache_v, draft_k, draft_v, path_nodes, dest_pages, dest_slots,
                 request):
    """Write accepted draft K/V to preallocated physical destinations."""
    return torch.ops.branchcraft.commit_path_(
        cache_k, cache_v, draft_k, draft_v, path_nodes, dest_pages, dest_slots, request)


def commit_batch_(cache_k, cache_v, draft_k, draft_v, clone_src, clone_dst, entry_request,
                  entry_node, entry_page, entry_slot):
    """All page clones of a commit plan, then all of its node writes."""
    return torch.ops.branchcraft.commit_batch_(
        cache_k, cache_v, draft_k, draft_v, clone_src, clone_dst, entry_request, entry_node,
        entry_page, entry_slot)
