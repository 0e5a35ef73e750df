"""ctypes binding of libbranchcraft.so (the C ABI of include/branchcraft.h).

Tensors are torch CUDA tensors; the binding passes their data pointers and the
current CUDA stream. Every call raises ``BranchcraftError`` on a non-zero
return code. There is no fallback: if the library is missing, importing this
module fails.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "lib" / "libbranchcraft.so"

if not LIB_PATH.exists():
    raise ImportError(f"branchcraft CUDA library missing: {LIB_PATH} (run the build)")

_lib = ctypes.CDLL(str(LIB_PATH))

PAGE_SIZE = 16
MAX_SPLITS = 64
MAX_NODES = 256
ERR_PAGE_RANGE, ERR_LENGTH, ERR_PARENT, ERR_TIMEOUT, ERR_COMMIT_INDEX = 1, 2, 4, 8, 16

EXPORTS = (
    "bc_decode", "bc_auto_splits", "bc_paged_decode", "bc_paged_decode_partial",
    "bc_tree_verify", "bc_tree_verify_f16", "bc_commit_path", "bc_commit_batch",
    "bc_packed_decode", "bc_packed_decode_kv", "bc_merge_partials",
    "bc_last_device_error", "bc_version", "bc_decode_static_scratch", "bc_merge_gathered",
    "bc_merge_to_partial", "bc_tree_verify_commit", "bc_selftest_bounded_wait",
    "bc_cow_plan", "bc_tree_step", "bc_exchange_bytes", "bc_exchange_create",
    "bc_exchange_open", "bc_exchange_close", "bc_exchange_destroy", "bc_merge_exchange",
)


class Shape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in
                ("batch", "query_heads", "kv_heads", "dim", "max_pages", "physical_pages")]


class BranchcraftError(RuntimeError):
    pass


_vp = ctypes.c_void_p
_i = ctypes.c_int
_ll = ctypes.c_longlong
_f = ctypes.c_float
_sz = ctypes.c_size_t
_SP = ctypes.POINTER(Shape)

_sigs = {
    "bc_decode": [_SP, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp],
    "bc_auto_splits": [_SP, _i, _i],
    "bc_paged_decode": [_SP, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp],
    "bc_paged_decode_partial": [_SP, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp],
    "bc_tree_verify": [_SP, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp],
    "bc_tree_verify_f16": [_SP, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp],
    "bc_commit_path": [_SP, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp],
    "bc_commit_batch": [_SP, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _vp],
    "bc_tree_verify_commit": [_SP, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i,
                              _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _vp],
    "bc_packed_decode": [_SP, _vp, _vp, _vp, _vp, _vp, _ll, _ll, _ll, _f, _vp],
    "bc_packed_decode_kv": [_SP, _vp, _vp, _vp, _vp, _vp, _ll, _ll, _ll, _ll, _f, _i, _vp],
    "bc_merge_partials": [_i, _i, _i, _vp, _vp, _vp, _vp],
    "bc_merge_gathered": [_i, _i, _i, _i, _vp, _vp, _vp],
    "bc_merge_to_partial": [_i, _i, _i, _vp, _vp, _vp, _vp, _vp],
    "bc_decode_static_scratch": [_SP, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp],
    "bc_selftest_bounded_wait": [_i, _i, ctypes.c_uint, _vp],
    "bc_cow_plan": [_i, _i, _i, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i,
                    _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "bc_tree_step": [_SP, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _vp, _vp, _vp,
                     _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                     _vp],
    "bc_exchange_bytes": [_i, _i, _i],
    "bc_exchange_create": [_i, _i, _i, ctypes.POINTER(_vp), _vp],
    "bc_exchange_open": [_vp, ctypes.POINTER(_vp)],
    "bc_exchange_close": [_vp],
    "bc_exchange_destroy": [_vp],
    "bc_merge_exchange": [_i, _i, ctypes.c_uint, _i, _i, _i, _vp, _vp, _vp, _vp, _vp],
    "bc_last_device_error": [_i],
    "bc_version": [],
}
for _name, _args in _sigs.items():
    _fn = getattr(_lib, _name)
    _fn.argtypes = _args
    _fn.restype = _i
_lib.bc_last_device_error.restype = ctypes.c_uint
_lib.bc_exchange_bytes.restype = _sz
_lib.bc_version.restype = ctypes.c_char_p


def lib():
    return _lib


def version() -> str:
    return _lib.bc_version().decode()


def _ptr(t):
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _check(rc: int, what: str):
    if rc != 0:
        raise BranchcraftError(f"{what} failed with cudaError {rc}")


def make_shape(batch, query_heads, kv_heads, dim, max_pages, physical_pages) -> Shape:
    return Shape(batch, query_heads, kv_heads, dim, max_pages, physical_pages)


def decode(shape: Shape, q, k, v, pages, lengths, output, partial_a=None, partial_ml=None,
           splits=1, stream=None, check=True):
    rc = _lib.bc_decode(ctypes.byref(shape), _ptr(q), _ptr(k), _ptr(v), _ptr(pages),
                        _ptr(lengths), _ptr(output), _ptr(partial_a), _ptr(partial_ml),
                        splits, _stream(stream))
    if check:
        _check(rc, "bc_decode")
    return rc


def auto_splits(shape: Shape, max_length: int, sm_count: int) -> int:
    return _lib.bc_auto_splits(ctypes.byref(shape), max_length, sm_count)


def paged_decode(shape, q, k, v, pages, lengths, output, splits=0, stream=None):
    _check(_lib.bc_paged_decode(ctypes.byref(shape), _ptr(q), _ptr(k), _ptr(v), _ptr(pages),
                                _ptr(lengths), _ptr(output), splits, _stream(stream)),
           "bc_paged_decode")


def paged_decode_partial(shape, q, k, v, pages, lengths, partial_ml, partial_a, splits=0,
                         stream=None):
    _check(_lib.bc_paged_decode_partial(ctypes.byref(shape), _ptr(q), _ptr(k), _ptr(v),
                                        _ptr(pages), _ptr(lengths), _ptr(partial_ml),
                                        _ptr(partial_a), splits, _stream(stream)),
           "bc_paged_decode_partial")


def tree_verify(shape, draft_q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent,
                output, nodes, stream=None):
    fn = _lib.bc_tree_verify_f16 if output.dtype == torch.float16 else _lib.bc_tree_verify
    _check(fn(ctypes.byref(shape), _ptr(draft_q), _ptr(prefix_k), _ptr(prefix_v), _ptr(pages),
              _ptr(lengths), _ptr(draft_k), _ptr(draft_v), _ptr(parent), _ptr(output), nodes,
              _stream(stream)), "bc_tree_verify")


def commit_path(shape, draft_k, draft_v, cache_k, cache_v, path_nodes, dest_pages, dest_slots,
                request, nodes, accepted, stream=None):
    _check(_lib.bc_commit_path(ctypes.byref(shape), _ptr(draft_k), _ptr(draft_v), _ptr(cache_k),
                               _ptr(cache_v), _ptr(path_nodes), _ptr(dest_pages),
                               _ptr(dest_slots), request, nodes, accepted, _stream(stream)),
           "bc_commit_path")


def commit_batch(shape, nodes, draft_k, draft_v, cache_k, cache_v, clone_src, clone_dst,
                 entry_request, entry_node, entry_page, entry_slot, stream=None):
    nclones = 0 if clone_src is None else int(clone_src.numel())
    nentries = 0 if entry_node is None else int(entry_node.numel())
    _check(_lib.bc_commit_batch(ctypes.byref(shape), nodes, _ptr(draft_k), _ptr(draft_v),
                                _ptr(cache_k), _ptr(cache_v), _ptr(clone_src), _ptr(clone_dst),
                                nclones, _ptr(entry_request), _ptr(entry_node),
                                _ptr(entry_page), _ptr(entry_slot), nentries, _stream(stream)),
           "bc_commit_batch")


def tree_verify_commit(shape, draft_q, cache_k, cache_v, pages, lengths, draft_k, draft_v,
                       parent, output, nodes, clone_src, clone_dst, entry_request, entry_node,
                       entry_page, entry_slot, stream=None):
    """tree_verify and the batch copy-on-write commit in one launch (the
    commit plan must be a copy-on-write plan: see bc_tree_verify_commit)."""
    nclones = 0 if clone_src is None else int(clone_src.numel())
    nentries = 0 if entry_node is None else int(entry_node.numel())
    _check(_lib.bc_tree_verify_commit(
        ctypes.byref(shape), _ptr(draft_q), _ptr(cache_k), _ptr(cache_v), _ptr(pages),
        _ptr(lengths), _ptr(draft_k), _ptr(draft_v), _ptr(parent), _ptr(output),
        1 if output.dtype == torch.float16 else 0, nodes, _ptr(clone_src), _ptr(clone_dst),
        nclones, _ptr(entry_request), _ptr(entry_node), _ptr(entry_page), _ptr(entry_slot),
        nentries, _stream(stream)), "bc_tree_verify_commit")


class CowPlan:
    """Device buffers of one batch's commit plan (capacities: `batch` clones,
    `batch * nodes` entries) and the page tables after the commit."""

    def __init__(self, batch, nodes, max_pages_out, device="cuda"):
        i32 = dict(device=device, dtype=torch.int32)
        self.batch, self.nodes, self.max_pages_out = batch, nodes, max_pages_out
        self.pages_out = torch.empty(batch, max_pages_out, **i32)
        self.lengths_out = torch.empty(batch, **i32)
        self.clone_src = torch.empty(batch, **i32)
        self.clone_dst = torch.empty(batch, **i32)
        self.entry_request = torch.empty(batch * nodes, **i32)
        self.entry_node = torch.empty(batch * nodes, **i32)
        self.entry_page = torch.empty(batch * nodes, **i32)
        self.entry_slot = torch.empty(batch * nodes, **i32)
        self.counts = torch.zeros(5, **i32)  # clones, entries, status, publication flag, arrivals

    def args(self):
        return (_ptr(self.pages_out), self.max_pages_out, _ptr(self.lengths_out),
                _ptr(self.clone_src), _ptr(self.clone_dst), _ptr(self.entry_request),
                _ptr(self.entry_node), _ptr(self.entry_page), _ptr(self.entry_slot),
                _ptr(self.counts))


def _state(state_in, state_out):
    """(refcount, free_stack, free_count) in and out: out defaults to in (an
    update in place)."""
    state_out = state_out if state_out is not None else state_in
    return tuple(_ptr(t) for t in state_in) + tuple(_ptr(t) for t in state_out)


def cow_plan(pages, lengths, path_len, path_nodes, state_in, plan: CowPlan, physical_pages,
             state_out=None, stream=None):
    """bc_cow_plan: the batch's copy-on-write bookkeeping on the device.
    state_in / state_out: (refcount, free_stack, free_count) tensors."""
    batch, max_pages_in = pages.shape
    (po, mpo, lo, cs, cd, er, en, ep, es, cnt) = plan.args()
    _check(_lib.bc_cow_plan(batch, plan.nodes, physical_pages, _ptr(pages), max_pages_in,
                            _ptr(lengths), _ptr(path_len), _ptr(path_nodes),
                            *_state(state_in, state_out), po, mpo, lo, cs, cd, er, en, ep, es,
                            cnt, _stream(stream)), "bc_cow_plan")


def tree_step(shape, draft_q, cache_k, cache_v, pages, lengths, draft_k, draft_v, parent,
              output, nodes, path_len, path_nodes, state_in, plan: CowPlan, state_out=None,
              stream=None):
    """bc_tree_step: device planner, then verify + commit in one launch."""
    (po, mpo, lo, cs, cd, er, en, ep, es, cnt) = plan.args()
    _check(_lib.bc_tree_step(ctypes.byref(shape), _ptr(draft_q), _ptr(cache_k), _ptr(cache_v),
                             _ptr(pages), _ptr(lengths), _ptr(draft_k), _ptr(draft_v),
                             _ptr(parent), _ptr(output), 1 if output.dtype == torch.float16 else 0,
                             nodes, _ptr(path_len), _ptr(path_nodes), *_state(state_in, state_out),
                             po, mpo, lo, cs, cd, er, en, ep, es, cnt, _stream(stream)),
           "bc_tree_step")


def packed_decode(shape, q, packed_kv, pages, lengths, output, block_stride, head_stride,
                  slot_stride, scale, stream=None):
    _check(_lib.bc_packed_decode(ctypes.byref(shape), _ptr(q), _ptr(packed_kv), _ptr(pages),
                                 _ptr(lengths), _ptr(output), block_stride, head_stride,
                                 slot_stride, scale, _stream(stream)), "bc_packed_decode")


def packed_decode_kv(shape, q, packed_kv, pages, lengths, output, block_stride, head_stride,
                     slot_stride, kv_offset, scale, splits=0, stream=None):
    _check(_lib.bc_packed_decode_kv(ctypes.byref(shape), _ptr(q), _ptr(packed_kv), _ptr(pages),
                                    _ptr(lengths), _ptr(output), block_stride, head_stride,
                                    slot_stride, kv_offset, scale, splits, _stream(stream)),
           "bc_packed_decode_kv")


def merge_partials(partial_ml, partial_a, out, stream=None):
    splits, rows, dim = partial_a.shape
    _check(_lib.bc_merge_partials(splits, rows, dim, _ptr(partial_ml), _ptr(partial_a),
                                  _ptr(out), _stream(stream)), "bc_merge_partials")


def exchange_bytes(world, rows, dim) -> int:
    return int(_lib.bc_exchange_bytes(world, rows, dim))


def exchange_create(world, rows, dim):
    """This rank's exchange buffer (device pointer, int) and its CUDA IPC
    handle (64 bytes) for the peers."""
    buf = _vp()
    handle = ctypes.create_string_buffer(64)
    _check(_lib.bc_exchange_create(world, rows, dim, ctypes.byref(buf), handle),
           "bc_exchange_create")
    return int(buf.value), handle.raw


def exchange_open(handle: bytes) -> int:
    """A peer's exchange buffer mapped into this process (device pointer)."""
    ptr = _vp()
    h = ctypes.create_string_buffer(bytes(handle), 64)
    _check(_lib.bc_exchange_open(h, ctypes.byref(ptr)), "bc_exchange_open")
    return int(ptr.value)


def exchange_close(ptr: int):
    _check(_lib.bc_exchange_close(_vp(ptr)), "bc_exchange_close")


def exchange_destroy(ptr: int):
    _check(_lib.bc_exchange_destroy(_vp(ptr)), "bc_exchange_destroy")


def merge_exchange(world, rank, epoch, partial_ml, partial_a, peers, out, stream=None):
    """bc_merge_exchange: partial_ml [S, rows, 2], partial_a [S, rows, dim]
    (this rank's split partials), peers: int64 device tensor of the world's
    exchange buffers in rank order; out [rows, dim] receives the merge of
    every rank's partials."""
    splits, rows, dim = partial_a.shape
    _check(_lib.bc_merge_exchange(world, rank, epoch, splits, rows, dim, _ptr(partial_ml),
                                  _ptr(partial_a), _ptr(peers), _ptr(out), _stream(stream)),
           "bc_merge_exchange")


def merge_to_partial(partial_ml, partial_a, out_ml, out_a, stream=None):
    """Merge [S, rows, *] partials into ONE partial per row: (M, L) into
    out_ml [rows, 2], the unnormalised accumulator into out_a [rows, dim]."""
    splits, rows, dim = partial_a.shape
    _check(_lib.bc_merge_to_partial(splits, rows, dim, _ptr(partial_ml), _ptr(partial_a),
                                    _ptr(out_ml), _ptr(out_a), _stream(stream)),
           "bc_merge_to_partial")


def merge_gathered(gathered, world, splits, rows, dim, out, stream=None):
    """Merge of `world` ranks' partial buffers gathered into one tensor
    ([world, splits*rows*(2+dim)]: each rank's (m, l) pairs, then its
    accumulators)."""
    _check(_lib.bc_merge_gathered(world, splits, rows, dim, _ptr(gathered), _ptr(out),
                                  _stream(stream)), "bc_merge_gathered")


def decode_static_scratch(shape: Shape, q, k, v, pages, lengths, output, splits=1,
                          stream=None, check=True):
    """bc_decode with the split partials in the library's fixed device array
    (no caller scratch, nothing allocated)."""
    rc = _lib.bc_decode_static_scratch(ctypes.byref(shape), _ptr(q), _ptr(k), _ptr(v),
                                       _ptr(pages), _ptr(lengths), _ptr(output), splits,
                                       _stream(stream))
    if check:
        _check(rc, "bc_decode_static_scratch")
    return rc


def selftest_bounded_wait(ctas, smem_bytes, limit_us, stream=None):
    _check(_lib.bc_selftest_bounded_wait(ctas, smem_bytes, limit_us, _stream(stream)),
           "bc_selftest_bounded_wait")


def last_device_error(reset: bool = True) -> int:
    return int(_lib.bc_last_device_error(1 if reset else 0))
