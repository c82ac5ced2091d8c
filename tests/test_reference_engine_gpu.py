"""The CUDA backend under the reference engine's own runtime: the reference's
tiny CNN (Conv -> BatchNorm -> Relu -> MaxPool -> Conv -> Relu ->
GlobalAvgPool -> Flatten -> Gemm, tests/golden/tiny_cnn.onnx) loaded by the
reference ONNX loader and run by

  * the reference Engine on its CPU backend,
  * BackendEngine with EngineConfig::gpu_backend = CUDA, which takes the CUDA
    backend from the reference BackendRegistry (compile() fuses BatchNorm and
    Relu into the convolutions, execute_async() keeps every value on the GPU),
  * CudaTraditionalEngine's infer() and batched infer_batch().

Bars: the ONNX Runtime logits of the reference's test
(tiny_cnn_reference.h) within 1e-3 * max |ref| (and the reference test's own
1e-4 absolute), the CPU engine within the same bound, repeated and batched
runs bit-identical to single runs."""
import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
HARNESS = ROOT / "oracle" / "_ref" / "ref_engine_harness"
GOLDEN = ROOT / "tests" / "golden"


@pytest.mark.skipif(not HARNESS.exists(), reason="reference engine harness not built")
def test_tiny_cnn_on_cuda_backend_matches_reference(tmp_path):
    g = json.loads((GOLDEN / "tiny_cnn.json").read_text())
    x = np.array(g["kTinyCnnInput"]["values"], np.float32)
    want = np.array(g["kTinyCnnExpected"]["values"], np.float32)
    inp = tmp_path / "x.f32"
    x.tofile(inp)
    r = subprocess.run([str(HARNESS), "gpu", str(GOLDEN / "tiny_cnn.onnx"), str(inp)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    res = json.loads(r.stdout.strip().splitlines()[-1])
    cuda = np.array(res["cuda"], np.float32)
    cpu = np.array(res["cpu"], np.float32)
    scale = float(np.abs(want).max())
    assert cuda.shape == want.shape
    assert np.abs(cuda - want).max() <= 1e-3 * scale
    assert np.abs(cuda - want).max() <= 1e-4          # the reference test's bound
    assert np.abs(cpu - want).max() <= 1e-4           # the reference engine itself
    assert np.abs(cuda - cpu).max() <= 1e-3 * scale
    assert res["cuda_again"] == res["cuda"]           # weights stay valid across runs
    assert res["single0"] == res["cuda"]
    assert res["batch0"] == res["single0"] and res["batch1"] == res["single1"]
    assert res["single1"] != res["single0"]
    assert res["folded_bn"] >= 1 and res["fused_act"] >= 1
