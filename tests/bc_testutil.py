"""Helpers shared by the test modules: moving oracle fixtures to the GPU and
seeded generators for the BASELINE-style configurations."""
from __future__ import annotations

import hashlib
import math
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_cases.npz"

DECODE_CASES = [
    (1, 8, 2, 64, [0]), (1, 8, 2, 64, [1]), (1, 8, 2, 64, [16]), (1, 8, 2, 64, [17]),
    (3, 10, 2, 64, [0, 37, 91]), (3, 12, 3, 128, [7, 128, 257]),
    (2, 32, 8, 128, [513, 3]),
]
TREE_CASES = [(0, 64, 31), (17, 64, 31), (257, 128, 31), (17, 128, 49)]


def golden():
    return np.load(GOLDEN)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def to_dev(a, device="cuda"):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.float16).to(device)
    return torch.from_numpy(a.copy()).to(device)


def half_bits(t) -> np.ndarray:
    """uint16 bit patterns of an FP16 torch tensor (any device)."""
    import torch

    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def rand_half(rng: np.random.Generator, shape, scale=1.0) -> np.ndarray:
    return (rng.standard_normal(shape, dtype=np.float32) * scale).astype(np.float16).view(np.uint16)


def random_tree_parents(rng: np.random.Generator, batch: int, nodes: int) -> np.ndarray:
    """parent[0] = -1, parent[i] uniform in [0, i-1]."""
    par = np.empty((batch, nodes), np.int32)
    par[:, 0] = -1
    for i in range(1, nodes):
        par[:, i] = rng.integers(0, i, size=batch)
    return par


def binary_tree_parents(batch: int, nodes: int) -> np.ndarray:
    par = np.array([-1] + [(n - 1) // 2 for n in range(1, nodes)], np.int32)
    return np.tile(par, (batch, 1))


def paged_fixture(rng, batch, hq, hkv, dim, lengths, pool_pages=None, shared_prefix=False,
                  scale=1.0):
    """Seeded paged K/V fixture with a random physical page permutation.

    shared_prefix: every request maps the same physical pages (lengths equal).
    """
    lengths = np.asarray(lengths, np.int32)
    npages = [(int(n) + 15) // 16 for n in lengths]
    max_pages = max(1, max(npages))
    used = npages[0] if shared_prefix else sum(npages)
    pool = pool_pages if pool_pages is not None else used + 7
    assert pool >= used
    perm = rng.permutation(pool).astype(np.int32)
    pages = np.full((batch, max_pages), -1, np.int32)
    cur = 0
    for b in range(batch):
        if shared_prefix:
            pages[b, :npages[b]] = perm[:npages[b]]
        else:
            pages[b, :npages[b]] = perm[cur:cur + npages[b]]
            cur += npages[b]
    k = rand_half(rng, (pool, 16, hkv, dim), scale)
    v = rand_half(rng, (pool, 16, hkv, dim), scale)
    q = rand_half(rng, (batch, hq, dim), scale)
    return dict(shape=(batch, hq, hkv, dim, max_pages, pool), q=q, k=k, v=v, pages=pages,
                lengths=lengths)


def max_abs(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    if not (np.isfinite(a).all() and np.isfinite(b).all()):
        return math.inf
    return float(np.abs(a - b).max()) if a.size else 0.0


def assert_close_baseline(actual, expected, atol=2e-3, rtol=1e-2):
    """The BASELINE tolerance: |a - e| <= atol + rtol * |e| elementwise."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert np.isfinite(a).all(), "non-finite output"
    bad = np.abs(a - e) > atol + rtol * np.abs(e)
    assert not bad.any(), f"{bad.sum()} elements outside atol={atol} rtol={rtol}; " \
                          f"max abs err {np.abs(a - e).max():.3e}"
