"""ctypes wrapper of the CPU oracle (oracle/liboracle.so) and, where it was
built, of the reference-built library (oracle/_ref/libbcref.so).

TEST INFRASTRUCTURE ONLY: imported by the pytest suite, the smoke check and
bench.py's CPU-baseline leg. FP16 arrays are numpy ``uint16`` bit patterns or
``float16`` arrays (same bytes).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_PATH = HERE / "_ref" / "libbcref.so"

PAGE = 16


class Shape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in
                ("batch", "query_heads", "kv_heads", "dim", "max_pages", "physical_pages")]

    def tuple(self):
        return (self.batch, self.query_heads, self.kv_heads, self.dim,
                self.max_pages, self.physical_pages)


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"oracle library missing: {LIB_PATH} (run make -C oracle)")
        _lib = ctypes.CDLL(str(LIB_PATH))
        _lib.bco_h2f.restype = ctypes.c_float
        _lib.bco_h2f.argtypes = [ctypes.c_uint16]
        _lib.bco_f2h.restype = ctypes.c_uint16
        _lib.bco_f2h.argtypes = [ctypes.c_float]
        _lib.bco_max_threads.restype = ctypes.c_int
    return _lib


def ref_available() -> bool:
    return REF_PATH.exists()


def ref():
    global _ref
    if _ref is None:
        if not REF_PATH.exists():
            raise ImportError(f"reference-built library missing: {REF_PATH}")
        _ref = ctypes.CDLL(str(REF_PATH))
    return _ref


def _u16(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    assert a.dtype == np.uint16, a.dtype
    return a


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def max_threads() -> int:
    return int(lib().bco_max_threads())


def f2h(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().bco_f2h_array(_p(x), _p(out), ctypes.c_longlong(x.size))
    return out


def h2f(x: np.ndarray) -> np.ndarray:
    x = _u16(x)
    out = np.empty(x.shape, np.float32)
    lib().bco_h2f_array(_p(x), _p(out), ctypes.c_longlong(x.size))
    return out


# ---------------------------------------------------------------- fixtures

def ref_fixture(batch, hq, hkv, dim, lengths, seed=17):
    """Reference make_fixture (src/main.cu:48-79) reproduced by the oracle."""
    lengths = _i32(lengths)
    mp, phys = ctypes.c_int(), ctypes.c_int()
    if lib().bco_ref_fixture_shape(batch, _p(lengths), ctypes.byref(mp), ctypes.byref(phys)):
        raise ValueError("negative length")
    mp, phys = mp.value, phys.value
    q = np.empty((batch, hq, dim), np.uint16)
    k = np.empty((phys, PAGE, hkv, dim), np.uint16)
    v = np.empty_like(k)
    pages = np.empty((batch, mp), np.int32)
    lib().bco_ref_fixture(batch, hq, hkv, dim, _p(lengths), ctypes.c_uint32(seed),
                          _p(q), _p(k), _p(v), _p(pages))
    return dict(shape=Shape(batch, hq, hkv, dim, mp, phys), q=q, k=k, v=v,
                pages=pages, lengths=lengths)


def ref_tree_fixture(batch, prefix_len, nodes, dim, seed=31):
    """Reference make_tree_fixture (src/main.cu:145-179) reproduced by the oracle."""
    s = Shape()
    lib().bco_ref_tree_fixture_shape(batch, prefix_len, ctypes.byref(s))
    s.dim = dim
    q = np.empty((batch, 32, dim), np.uint16)
    k = np.empty((s.physical_pages, PAGE, 8, dim), np.uint16)
    v = np.empty_like(k)
    pages = np.empty((batch, s.max_pages), np.int32)
    lengths = np.empty(batch, np.int32)
    dq = np.empty((batch, nodes, 32, dim), np.uint16)
    dk = np.empty((batch, nodes, 8, dim), np.uint16)
    dv = np.empty_like(dk)
    parent = np.empty((batch, nodes), np.int32)
    if lib().bco_ref_tree_fixture(batch, prefix_len, nodes, dim, ctypes.c_uint32(seed),
                                  _p(q), _p(k), _p(v), _p(pages), _p(lengths),
                                  _p(dq), _p(dk), _p(dv), _p(parent)):
        raise ValueError("bad tree fixture")
    return dict(shape=s, q=q, k=k, v=v, pages=pages, lengths=lengths, nodes=nodes,
                draft_q=dq, draft_k=dk, draft_v=dv, parent=parent)


# ---------------------------------------------------------------- oracles

def decode(shape, q, k, v, pages, lengths, threads=0):
    """Paged GQA decode oracle (src/main.cu:81-113). FP32 [B,Hq,D]."""
    s = Shape(*shape) if not isinstance(shape, Shape) else shape
    q, k, v = _u16(q), _u16(k), _u16(v)
    pages, lengths = _i32(pages), _i32(lengths)
    out = np.empty((s.batch, s.query_heads, s.dim), np.float32)
    lib().bco_decode(ctypes.byref(s), _p(q), _p(k), _p(v), _p(pages), _p(lengths),
                     _p(out), threads)
    return out


def tree(shape, nodes, draft_q, k, v, pages, lengths, draft_k, draft_v, parent,
         threads=0):
    """Tree-verify oracle (src/main.cu:204-240). FP32 [B,N,Hq,D]."""
    s = Shape(*shape) if not isinstance(shape, Shape) else shape
    arrs = [_u16(draft_q), _u16(k), _u16(v), _i32(pages), _i32(lengths),
            _u16(draft_k), _u16(draft_v), _i32(parent)]
    out = np.empty((s.batch, nodes, s.query_heads, s.dim), np.float32)
    rc = lib().bco_tree(ctypes.byref(s), nodes, *[_p(a) for a in arrs], _p(out), threads)
    if rc:
        raise ValueError("parent chains leave [0, nodes) or are cyclic")
    return out


def packed_decode(shape, q, cache, pages, lengths, block_stride, head_stride,
                  slot_stride, kv_offset, scale, threads=0, want_f32=False):
    """Packed-cache decode oracle (tests/test_torch_ops.py:77-88). FP16 [B,Hq,D]."""
    s = Shape(*shape) if not isinstance(shape, Shape) else shape
    q, cache = _u16(q), _u16(cache)
    pages, lengths = _i32(pages), _i32(lengths)
    out = np.empty((s.batch, s.query_heads, s.dim), np.uint16)
    f32 = np.empty((s.batch, s.query_heads, s.dim), np.float32) if want_f32 else None
    lib().bco_packed_decode(ctypes.byref(s), _p(q), _p(cache), _p(pages), _p(lengths),
                            ctypes.c_longlong(block_stride), ctypes.c_longlong(head_stride),
                            ctypes.c_longlong(slot_stride), ctypes.c_longlong(kv_offset),
                            ctypes.c_float(scale), _p(out), _p(f32), threads)
    return (out, f32) if want_f32 else out


def commit(cache_k, cache_v, draft_k, draft_v, path_nodes, dest_pages, dest_slots,
           request):
    """commit_path oracle (src/tree_attention.cu:73-89); updates caches in place."""
    assert cache_k.flags.c_contiguous and cache_v.flags.c_contiguous
    ck, cv = cache_k.view(np.uint16), cache_v.view(np.uint16)
    dk, dv = _u16(draft_k), _u16(draft_v)
    path, dp, ds = _i32(path_nodes), _i32(dest_pages), _i32(dest_slots)
    P, _, hkv, dim = ck.shape
    nodes = dk.shape[1]
    rc = lib().bco_commit(hkv, dim, P, nodes, _p(dk), _p(dv), _p(ck), _p(cv),
                          _p(path), _p(dp), _p(ds), request, len(path))
    if rc:
        raise ValueError("commit index out of range")


def merge(partial_ml, partial_a):
    """FP32 split merge (src/paged_gqa.cu:76-106). partial_ml [S,rows,2], partial_a [S,rows,D]."""
    pml = np.ascontiguousarray(partial_ml, np.float32)
    pa = np.ascontiguousarray(partial_a, np.float32)
    S, rows, dim = pa.shape
    out = np.empty((rows, dim), np.float32)
    lib().bco_merge(S, rows, dim, _p(pml), _p(pa), _p(out))
    return out


# ------------------------------------------------------- reference-built lib

def ref_make_fixture(batch, hq, hkv, dim, lengths, seed=17):
    r = ref()
    lengths = _i32(lengths)
    s = Shape()
    if r.bcr_make_fixture(batch, hq, hkv, dim, _p(lengths), ctypes.c_uint32(seed),
                          ctypes.byref(s), None, None, None, None):
        raise ValueError("reference fixture failed")
    q = np.empty((batch, hq, dim), np.uint16)
    k = np.empty((s.physical_pages, PAGE, hkv, dim), np.uint16)
    v = np.empty_like(k)
    pages = np.empty((batch, s.max_pages), np.int32)
    r.bcr_make_fixture(batch, hq, hkv, dim, _p(lengths), ctypes.c_uint32(seed),
                       ctypes.byref(s), _p(q), _p(k), _p(v), _p(pages))
    return dict(shape=s, q=q, k=k, v=v, pages=pages, lengths=lengths)


def ref_cpu_reference(shape, q, k, v, pages, lengths):
    s = Shape(*shape) if not isinstance(shape, Shape) else shape
    out = np.empty((s.batch, s.query_heads, s.dim), np.float32)
    ref().bcr_cpu_reference(ctypes.byref(s), _p(_u16(q)), _p(_u16(k)), _p(_u16(v)),
                            _p(_i32(pages)), _p(_i32(lengths)), _p(out))
    return out


def ref_make_tree_fixture(batch, prefix_len, nodes, dim, seed=31):
    r = ref()
    s = Shape()
    nulls = [None] * 9
    if r.bcr_make_tree_fixture(batch, prefix_len, nodes, dim, ctypes.c_uint32(seed),
                               ctypes.byref(s), *nulls):
        raise ValueError("reference tree fixture failed")
    q = np.empty((batch, 32, dim), np.uint16)
    k = np.empty((s.physical_pages, PAGE, 8, dim), np.uint16)
    v = np.empty_like(k)
    pages = np.empty((batch, s.max_pages), np.int32)
    lengths = np.empty(batch, np.int32)
    dq = np.empty((batch, nodes, 32, dim), np.uint16)
    dk = np.empty((batch, nodes, 8, dim), np.uint16)
    dv = np.empty_like(dk)
    parent = np.empty((batch, nodes), np.int32)
    r.bcr_make_tree_fixture(batch, prefix_len, nodes, dim, ctypes.c_uint32(seed),
                            ctypes.byref(s), _p(q), _p(k), _p(v), _p(pages), _p(lengths),
                            _p(dq), _p(dk), _p(dv), _p(parent))
    return dict(shape=s, q=q, k=k, v=v, pages=pages, lengths=lengths, nodes=nodes,
                draft_q=dq, draft_k=dk, draft_v=dv, parent=parent)


def ref_cpu_tree_reference(shape, nodes, draft_q, k, v, pages, lengths, draft_k,
                           draft_v, parent):
    s = Shape(*shape) if not isinstance(shape, Shape) else shape
    out = np.empty((s.batch, nodes, s.query_heads, s.dim), np.float32)
    ref().bcr_cpu_tree_reference(ctypes.byref(s), nodes, _p(_u16(draft_q)), _p(_u16(k)),
                                 _p(_u16(v)), _p(_i32(pages)), _p(_i32(lengths)),
                                 _p(_u16(draft_k)), _p(_u16(draft_v)), _p(_i32(parent)),
                                 _p(out))
    return out


if os.environ.get("BC_ORACLE_THREADS"):
    os.environ.setdefault("OMP_NUM_THREADS", os.environ["BC_ORACLE_THREADS"])
