"""The C++ ops behind the reference Op / OpRegistry interface, without a GPU:
attribute parsing and error codes as the reference's Conv2DOp tests assert
them (tests/unit/traditional_ops_test.cpp:195-222), registry semantics
(op_registry.cpp:23-50), and forward() failing with Runtime when no CUDA
device exists (no CPU fallback); the int8 quantizer's plugin contract and
error codes; the Conv + BatchNorm + Relu fusion pass on small graphs.  Also
compiles the op, quantizer and pass sources against the
reference's own headers when the reference tree is present, which shows they
drop into the reference engine unchanged."""
import os
import subprocess
from pathlib import Path

import pytest

from tests.backend_cpp import ROOT, driver

REFERENCE_SRC = Path("/root/reference/src")


def test_cpp_ops_configure_validate_registry():
    env = dict(os.environ)
    r = subprocess.run([str(driver()), "cpu"], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASSED" in r.stdout


@pytest.mark.skipif(not REFERENCE_SRC.exists(), reason="reference tree not present")
def test_cpp_ops_compile_against_reference_headers():
    backend = ROOT / "computeengine_b200" / "csrc" / "backend"
    cmd = ["g++", "-std=c++20", "-fsyntax-only", "-DIE_B200_REFERENCE_HEADERS",
           f"-I{REFERENCE_SRC}", f"-I{ROOT / 'include'}", f"-I{backend}",
           "-I/usr/local/cuda/include", str(backend / "cuda_conv_ops.cpp"),
           str(backend / "int8_quant.cpp"), str(backend / "graph_passes.cpp"),
           str(backend / "cuda_executor.cpp")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
