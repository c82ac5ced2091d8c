"""Build recipe for the native parts of the package (in-tree, sm_100a only).

    python -m computeengine_b200.build

produces computeengine_b200/libie_cuda_conv.so (CUDA kernels + C ABI) and
computeengine_b200/libie_cuda_backend.so (C++ engine-side backend: the
CudaConv2DOp / CudaDepthwiseConv2DOp ops and their registry), plus the C++
backend test driver under computeengine_b200/_build/.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libie_cuda_conv.so"
BACKEND_LIB = PKG / "libie_cuda_backend.so"
BUILD_DIR = PKG / "_build"
BACKEND_TEST = BUILD_DIR / "ie_cuda_backend_test"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _newer(target: Path, sources) -> bool:
    if not target.exists():
        return False
    t = target.stat().st_mtime
    return all(Path(s).stat().st_mtime <= t for s in sources)


def _run(cmd):
    print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def build_cuda(force: bool = False) -> Path:
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) \
        + [ROOT / "include" / "ie_cuda_conv.h"]
    if not force and _newer(LIB, sources):
        return LIB
    cuda_lib = Path(nvcc()).resolve().parent.parent / "lib64"
    _run([nvcc(), *NVCC_FLAGS, "-shared", "-o", LIB, CSRC / "ie_cuda_conv.cu",
          "-Xlinker", f"-rpath={cuda_lib}"])
    return LIB


def build_backend(force: bool = False) -> Path:
    """C++ engine-side backend, linked against the CUDA library."""
    bdir = CSRC / "backend"
    srcs = sorted(bdir.glob("*.cpp"))
    if not srcs:
        return BACKEND_LIB
    deps = srcs + sorted(bdir.glob("*.h")) + [LIB, ROOT / "include" / "ie_cuda_conv.h"]
    cuda_inc = Path(nvcc()).resolve().parent.parent / "include"
    cuda_lib = Path(nvcc()).resolve().parent.parent / "lib64"
    common = ["-O2", "-std=c++20", "-fPIC", f"-I{ROOT / 'include'}", f"-I{bdir}",
              f"-I{cuda_inc}"]
    if force or not _newer(BACKEND_LIB, deps):
        lib_srcs = [s for s in srcs if not s.name.endswith("_test.cpp")]
        _run(["g++", *common, "-shared", "-o", BACKEND_LIB, *lib_srcs, f"-L{PKG}",
              "-lie_cuda_conv", f"-L{cuda_lib}", "-lcudart", f"-Wl,-rpath,$ORIGIN",
              f"-Wl,-rpath,{cuda_lib}"])
    tests = [s for s in srcs if s.name.endswith("_test.cpp")]
    if tests and (force or not _newer(BACKEND_TEST, tests + [BACKEND_LIB])):
        BUILD_DIR.mkdir(exist_ok=True)
        _run(["g++", *common, "-o", BACKEND_TEST, *tests, f"-L{PKG}", "-lie_cuda_backend",
              "-lie_cuda_conv", f"-L{cuda_lib}", "-lcudart", f"-Wl,-rpath,{PKG}",
              f"-Wl,-rpath,{cuda_lib}"])
    return BACKEND_LIB


def build(force: bool = False) -> None:
    build_cuda(force)
    build_backend(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
