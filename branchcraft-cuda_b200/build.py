"""Build every native piece of the package in-tree.

    python branchcraft-cuda_b200/build.py [--force]

Products (all git-ignored, all shipped with the tree):
  lib/libbranchcraft.so       the CUDA kernels + C ABI (nvcc, sm_100a only)
  branchcraft_torch/_C.so     the TORCH_LIBRARY(branchcraft) binding (g++)
  ../tests/cli/branchcraft    the `branchcraft test | bench | tree-bench` driver
The CPU oracle (../oracle) is test infrastructure with its own Makefile; the
repository-level build entry point builds it too.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "lib" / "libbranchcraft.so"
TORCH_EXT = PKG / "branchcraft_torch" / "_C.so"
CLI_SRC = ROOT / "tests" / "cli" / "branchcraft_main.cpp"
CLI_BIN = ROOT / "tests" / "cli" / "branchcraft"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall"]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda) / "bin" / "nvcc"
    return str(cand) if cand.exists() else (shutil.which("nvcc") or "nvcc")


def _cxx() -> str:
    return shutil.which("g++") or "g++"


def _stale(target: Path, sources) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(s).stat().st_mtime > t for s in sources)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def build_library(force=False, verbose=True):
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "branchcraft.h"]
    if not force and not _stale(LIB, sources):
        return
    LIB.parent.mkdir(parents=True, exist_ok=True)
    _run([_nvcc(), *NVCC_FLAGS, *ARCH, "-shared", f"-I{INCLUDE}", f"-I{CSRC}",
          CSRC / "branchcraft.cu", "-o", LIB], verbose)


def build_torch_ext(force=False, verbose=True):
    src = CSRC / "torch_ops.cpp"
    if not force and not _stale(TORCH_EXT, [src, INCLUDE / "branchcraft.h", LIB]):
        return
    import torch
    from torch.utils.cpp_extension import include_paths, library_paths

    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [_cxx(), "-O2", "-std=c++17", "-fPIC", "-shared", str(src),
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
           f"-I{INCLUDE}", f"-I{cuda}/include"]
    cmd += [f"-I{p}" for p in include_paths()]
    cmd += [f"-L{LIB.parent}", "-lbranchcraft", "-Wl,-rpath,$ORIGIN/../lib"]
    for p in library_paths():
        cmd += [f"-L{p}", f"-Wl,-rpath,{p}"]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
            f"-L{cuda}/lib64", "-lcudart", "-o", str(TORCH_EXT)]
    _run(cmd, verbose)


def build_cli(force=False, verbose=True):
    """The reference-compatible driver; its `test` mode links the CPU oracle."""
    if not CLI_SRC.exists():
        return
    oracle_src = ROOT / "oracle" / "bc_oracle.cpp"
    sources = [CLI_SRC, oracle_src, INCLUDE / "branchcraft.h", INCLUDE / "branchcraft.hpp", LIB]
    if not force and not _stale(CLI_BIN, sources):
        return
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    _run([_cxx(), "-O2", "-std=c++17", "-fopenmp", str(CLI_SRC), str(oracle_src),
          f"-I{INCLUDE}", f"-I{cuda}/include", f"-L{LIB.parent}", "-lbranchcraft",
          "-Wl,-rpath,$ORIGIN/../../branchcraft-cuda_b200/lib", f"-L{cuda}/lib64", "-lcudart",
          f"-Wl,-rpath,{cuda}/lib64", "-o", str(CLI_BIN)], verbose)


def build_all(force=False, verbose=True):
    build_library(force, verbose)
    build_torch_ext(force, verbose)
    build_cli(force, verbose)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--quiet", action="store_true")
    a = ap.parse_args()
    build_all(a.force, not a.quiet)
    sys.exit(0)
