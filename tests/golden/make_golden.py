"""Generate tests/golden/reference_cases.npz from the reference itself.

Runs the reference's own fixture generators and CPU oracle (src/main.cu,
compiled unmodified into oracle/_ref/libbcref.so by `make -C oracle ref`) on
every known-answer case of the reference's `branchcraft test` driver:

* the 7 decode cases of src/main.cu:320-326 (seed 17),
* the 3 tree cases of src/main.cu:254 (B=2, 7 nodes, seed 31),
* the commit-scenario tree fixture of src/main.cu:267 (prefix 17, D=128, seed 49).

For each case it stores the SHA-256 of the generated input bytes (so a test
can prove its regenerated inputs are the reference's) and the reference's
FP32 output. Run from the repository root:

    make -C oracle && make -C oracle ref REF=<reference root>
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
import oracle as O  # noqa: E402

DECODE_CASES = [
    (1, 8, 2, 64, [0]), (1, 8, 2, 64, [1]), (1, 8, 2, 64, [16]), (1, 8, 2, 64, [17]),
    (3, 10, 2, 64, [0, 37, 91]), (3, 12, 3, 128, [7, 128, 257]),
    (2, 32, 8, 128, [513, 3]),
]
TREE_CASES = [(0, 64, 31), (17, 64, 31), (257, 128, 31), (17, 128, 49)]


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main() -> None:
    if not O.ref_available():
        raise SystemExit("oracle/_ref/libbcref.so is missing; build it with make -C oracle ref")
    out = {}
    for i, (b, hq, hkv, d, lens) in enumerate(DECODE_CASES):
        f = O.ref_make_fixture(b, hq, hkv, d, lens, 17)
        res = O.ref_cpu_reference(f["shape"], f["q"], f["k"], f["v"], f["pages"], f["lengths"])
        out[f"decode{i}_spec"] = np.array([b, hq, hkv, d] + list(f["shape"].tuple()), np.int32)
        out[f"decode{i}_lengths"] = np.array(lens, np.int32)
        out[f"decode{i}_sha"] = np.array(digest(f["q"], f["k"], f["v"], f["pages"]))
        out[f"decode{i}_out"] = res
    for i, (prefix, d, seed) in enumerate(TREE_CASES):
        f = O.ref_make_tree_fixture(2, prefix, 7, d, seed)
        res = O.ref_cpu_tree_reference(f["shape"], 7, f["draft_q"], f["k"], f["v"], f["pages"],
                                       f["lengths"], f["draft_k"], f["draft_v"], f["parent"])
        out[f"tree{i}_spec"] = np.array([prefix, d, seed] + list(f["shape"].tuple()), np.int32)
        out[f"tree{i}_sha"] = np.array(digest(f["q"], f["k"], f["v"], f["pages"], f["lengths"],
                                              f["draft_q"], f["draft_k"], f["draft_v"],
                                              f["parent"]))
        out[f"tree{i}_out"] = res
    dst = Path(__file__).resolve().parent / "reference_cases.npz"
    np.savez_compressed(dst, **out)
    print(f"wrote {dst} ({dst.stat().st_size} bytes, {len(DECODE_CASES)} decode + "
          f"{len(TREE_CASES)} tree cases)")


if __name__ == "__main__":
    main()
