"""Failure detection of the kernels' bounded waits, exercised without a GPU
fault: a self-test kernel waits on an mbarrier that nothing arrives on, with
a 1 ms limit passed at launch.  The wait gives up, the device error word holds
the probe's code, the kernel frees its tensor memory and returns, and the
context stays usable: a convolution run right after it is bit-exact."""
import ctypes

import numpy as np
import pytest

from tests.qconv import make_q8_problem, run_conv_q8_gpu

pytestmark = pytest.mark.gpu

PROBE_CODE = 0x1FF


def test_bounded_wait_gives_up_and_context_survives(oracle):
    import torch
    from computeengine_b200 import _lib as L
    assert L.take_device_error() == 0
    stream = torch.cuda.current_stream().cuda_stream
    waited = ctypes.c_uint64(0)
    L.check(L.lib.ie_cuda_bounded_wait_probe(1_000_000, waited, stream))  # 1 ms limit
    assert 1_000_000 <= waited.value < 200_000_000, waited.value
    assert L.take_device_error() == PROBE_CODE
    assert L.take_device_error() == 0  # reading clears it
    # twice in a row: tensor memory was freed by the first probe
    L.check(L.lib.ie_cuda_bounded_wait_probe(200_000, waited, stream))
    assert L.take_device_error() == PROBE_CODE
    rng = np.random.default_rng(12)
    x, wq, bias, mult = make_q8_problem(rng, 2, 64, 12, 12, 128, 3, 3, s_y=0.05 * 24 * 3)
    got = run_conv_q8_gpu(x, wq, bias, mult, pads=(1, 1, 1, 1))
    np.testing.assert_array_equal(got, oracle.conv2d_q8(x, wq, bias, mult, 128, 0, 0, 255,
                                                        pads=(1, 1, 1, 1)))


def test_probe_rejects_unbounded_limits():
    from computeengine_b200 import _lib as L
    assert L.lib.ie_cuda_bounded_wait_probe(0, None, None) == L.IE_INVALID_ARGUMENT
    assert L.lib.ie_cuda_bounded_wait_probe(3_000_000_000, None, None) == L.IE_INVALID_ARGUMENT
