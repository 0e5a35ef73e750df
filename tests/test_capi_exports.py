"""The C-ABI library loads without a GPU and exports every entry point that
include/branchcraft.h declares; the C++ header compiles against it."""
import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "branchcraft.h"
LIB = ROOT / "branchcraft-cuda_b200" / "lib" / "libbranchcraft.so"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|unsigned|size_t|const char\*)\s+(bc_\w+)\s*\(",
                                 text, re.M)))


def test_header_declares_the_boundary():
    names = declared()
    for n in ("bc_decode", "bc_auto_splits", "bc_tree_verify", "bc_commit_path",
              "bc_packed_decode"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(LIB))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_module_loads_and_matches_header():
    import bc_capi

    assert set(bc_capi.EXPORTS) == set(declared())
    assert "sm_100a" in bc_capi.version()


def test_host_side_argument_rejection_needs_no_gpu():
    """Argument validation happens before any device call (reference rules)."""
    import bc_capi as C

    lib = C.lib()
    bad = C.make_shape(1, 8, 2, 96, 1, 1)
    assert lib.bc_decode(ctypes.byref(bad), None, None, None, None, None, None, None, None, 1,
                         None) == 1
    ok_shape = C.make_shape(1, 8, 2, 64, 1, 1)
    # null scratch with splits > 1
    p = ctypes.c_void_p(16)
    assert lib.bc_decode(ctypes.byref(ok_shape), p, p, p, p, p, p, None, None, 2, None) == 1
    assert lib.bc_decode(ctypes.byref(ok_shape), p, p, p, p, p, p, None, None, 65, None) == 1
    assert lib.bc_tree_verify(ctypes.byref(ok_shape), p, p, p, p, p, p, p, p, p, 257, None) == 1
    assert lib.bc_commit_path(ctypes.byref(ok_shape), p, p, p, p, p, p, p, 1, 3, 1, None) == 1
    assert lib.bc_packed_decode(ctypes.byref(ok_shape), p, p, p, p, p, 4096, 2048, 128,
                                ctypes.c_float(0.0), None) == 1
    assert C.auto_splits(ok_shape, 100, 148) == 1


@pytest.mark.skipif(shutil.which("g++") is None, reason="no host compiler")
def test_cpp_header_is_a_drop_in(tmp_path):
    """Code written against the reference header compiles and links unchanged."""
    src = tmp_path / "user.cpp"
    src.write_text(r'''
#include "branchcraft.hpp"
int main() {
  branchcraft::Shape s{1, 8, 2, 64, 1, 1};
  branchcraft::Inputs in{};
  branchcraft::Scratch scratch{nullptr, nullptr};
  cudaError_t e = branchcraft::decode(s, in, scratch, 1);
  branchcraft::TreeInputs t{};
  e = branchcraft::tree_verify(s, t, 7);
  e = branchcraft::commit_path(s, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                               nullptr, 0, 7, 3);
  e = branchcraft::packed_decode(s, nullptr, nullptr, nullptr, nullptr, nullptr, 1, 1, 1, 1.f);
  int sp = branchcraft::auto_splits(s, 4096, 148);
  return (e == cudaErrorInvalidValue && sp >= 1 && branchcraft::kPageSize == 16) ? 0 : 1;
}
''')
    exe = tmp_path / "user"
    subprocess.run(["g++", "-std=c++17", str(src), f"-I{ROOT / 'include'}",
                    "-I/usr/local/cuda/include", f"-L{LIB.parent}", "-lbranchcraft",
                    f"-Wl,-rpath,{LIB.parent}", "-o", str(exe)], check=True)
    assert subprocess.run([str(exe)]).returncode == 0
