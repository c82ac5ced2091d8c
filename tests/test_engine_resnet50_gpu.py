"""The int8 ResNet-50 as one engine graph through the C++ CudaExecutor
(the reference Executor's interface, src/core/runtime/executor.cpp:53-83):
53 quantized Conv2D nodes, MaxPool2D, 16 int8 shortcut Adds, the int8
GlobalAvgPool, Flatten and the fp32 Gemm, run with host tensors in and out.
Every op on the way is checked against the oracle on its own in the other
GPU tests; here the whole graph must run, launch one kernel per node (plus
the input pack), hold only its live set of activations in the executor's
stream-ordered pool, and give image 0 alone the batch's first row of logits."""
import json
import subprocess

import pytest

from tests.backend_cpp import driver

pytestmark = pytest.mark.gpu


def _engine_bench(batch, iters, warmup):
    out = subprocess.run([str(driver()), "engine-bench", str(batch), str(iters), str(warmup)],
                         capture_output=True, text=True, timeout=600)
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert lines, out.stdout + out.stderr
    return out.returncode, json.loads(lines[-1])


def test_resnet50_q8_graph_runs_through_executor():
    rc, r = _engine_bench(4, 2, 1)
    assert rc == 0, r
    assert "error" not in r
    assert r["nodes"] == 53 + 1 + 16 + 3
    assert r["batch1_ok"] is True
    assert r["max_abs_logit"] > 0
    assert r["h2d_bytes_per_run"] == 4 * 3 * 224 * 224
    assert r["d2h_bytes_per_run"] == 4 * 1000 * 4
    # one launch per node at most (Flatten launches nothing), the graph
    # input's pack and the logits; no per-node copies
    assert 70 <= r["launches_per_run"] <= 80


def test_executor_pool_holds_the_live_set():
    """Released after their last reader, the activations of a batch-32 run
    fit in a fraction of the sum of all the graph's values (~540 MB at batch
    32 in the NHWC layout; the largest live set, around stage 1's first Add,
    is ~80 MB)."""
    rc, r = _engine_bench(32, 2, 1)
    assert rc == 0, r
    assert 0 < r["device_pool_reserved_bytes"] < 300 * 2**20
