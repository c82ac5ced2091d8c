"""Two devices in one process: the same kernel variants launch on device 0
and then on device 1 (the shared-memory opt-in and the no-allocation scratch
address are per device).  Plain single-device launches on each GPU, no peer
memory.  Skipped with fewer than two visible GPUs."""
import numpy as np
import pytest

from tests.qconv import make_q8_problem, run_conv_q8_gpu

pytestmark = pytest.mark.gpu


def _need_two():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two visible GPUs")


def test_int8_conv_on_two_devices(oracle):
    _need_two()
    import torch
    rng = np.random.default_rng(21)
    x, wq, bias, mult = make_q8_problem(rng, 2, 64, 16, 16, 128, 3, 3, s_y=0.05 * 24 * 3)
    want = oracle.conv2d_q8(x, wq, bias, mult, 128, 0, 0, 255, pads=(1, 1, 1, 1))
    prev = torch.cuda.current_device()
    try:
        for dev in (0, 1, 0):
            torch.cuda.set_device(dev)
            got = run_conv_q8_gpu(x, wq, bias, mult, pads=(1, 1, 1, 1), device=f"cuda:{dev}")
            np.testing.assert_array_equal(got, want)
    finally:
        torch.cuda.set_device(prev)


def test_noalloc_on_two_devices(oracle):
    _need_two()
    import torch
    from computeengine_b200 import _lib as L
    from tests.qconv import desc_for
    rng = np.random.default_rng(4)
    x = rng.uniform(-1, 1, (1, 32, 12, 12)).astype(np.float32)
    w = rng.normal(0, 0.1, (48, 32, 3, 3)).astype(np.float32)
    want = oracle.conv2d_f32(x, w, None, pads=(1, 1, 1, 1))
    d = desc_for(L, 1, 32, 12, 12, 48, 3, 3, (1, 1), (1, 1, 1, 1))
    prev = torch.cuda.current_device()
    try:
        for dev in (1, 0):
            torch.cuda.set_device(dev)
            xd = torch.from_numpy(x).cuda(dev)
            wd = torch.from_numpy(w).cuda(dev)
            y = torch.full((1, 48, 12, 12), float("nan"), device=f"cuda:{dev}")
            L.check(L.lib.ie_cuda_conv2d_f32_noalloc(d, 0, xd.data_ptr(), wd.data_ptr(), None,
                                                     y.data_ptr(),
                                                     torch.cuda.current_stream(dev).cuda_stream))
            torch.cuda.synchronize(dev)
            err = float(np.abs(y.cpu().numpy() - want).max())
            assert err <= 1e-3 * float(np.abs(want).max()), (dev, err)
    finally:
        torch.cuda.set_device(prev)
