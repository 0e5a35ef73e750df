"""The reference's own caller tests, run unchanged against this package.

`make -C oracle callers REF=<reference checkout>` (run by the repository's
build step where the reference is present) copies the reference's
tests/test_torch_ops.py (:17-113), tests/test_transaction.py (:8-29) and
tests/test_vllm_backend.py (:16-54) byte for byte into oracle/_ref/callers
(build output, not part of this repository's sources). Here they run in their
own pytest process with this package's branchcraft_torch and branchcraft_vllm
first on the import path: the drop-in contract is that a caller written
against the reference passes without edits.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
CALLERS = ROOT / "oracle" / "_ref" / "callers"
FILES = ("test_torch_ops.py", "test_transaction.py", "test_vllm_backend.py")


@pytest.mark.timeout(900)
def test_reference_callers_pass_unchanged():
    missing = [f for f in FILES if not (CALLERS / f).exists()]
    if missing:
        pytest.skip(f"reference caller tests not built into {CALLERS}: {missing}")
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join(
        [str(ROOT / "branchcraft-cuda_b200")] + [p for p in env.get("PYTHONPATH", "").split(
            os.pathsep) if p])
    r = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-rA",
         "--rootdir", str(CALLERS), "-c", os.devnull, *[str(CALLERS / f) for f in FILES]],
        cwd=str(CALLERS), env=env, capture_output=True, text=True, timeout=850)
    tail = (r.stdout + r.stderr)[-4000:]
    assert r.returncode == 0, tail
    assert " passed" in r.stdout and " failed" not in r.stdout and "skipped" not in r.stdout, tail
