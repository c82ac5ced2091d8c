"""The C++ ops behind the reference Op / OpRegistry interface, without a GPU:
attribute parsing and error codes as the reference's Conv2DOp tests assert
them (tests/unit/traditional_ops_test.cpp:195-222), registry semantics
(op_registry.cpp:23-50), and forward() failing with Runtime when no CUDA
device exists (no CPU fallback); the int8 quantizer's plugin contract and
error codes; the Conv + BatchNorm + Relu fusion pass on small graphs.  Also
runs the reference-engine harness (oracle/_ref/ref_engine_harness: the
backend sources compiled against the reference's own headers and linked with
its Engine, registries and ONNX loader) in its no-GPU mode: the CUDA backend
registers in the reference BackendRegistry and reports the missing device."""
import os
import subprocess
from pathlib import Path

import pytest

from tests.backend_cpp import ROOT, driver

HARNESS = ROOT / "oracle" / "_ref" / "ref_engine_harness"
TINY_CNN = ROOT / "tests" / "golden" / "tiny_cnn.onnx"


def test_cpp_ops_configure_validate_registry():
    env = dict(os.environ)
    r = subprocess.run([str(driver()), "cpu"], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASSED" in r.stdout


@pytest.mark.skipif(not HARNESS.exists(), reason="reference engine harness not built here")
def test_cuda_backend_registers_in_reference_runtime():
    r = subprocess.run([str(HARNESS), "cpu", str(TINY_CNN)], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASSED" in r.stdout
