"""1x1, stride-1, unpadded convolutions load their A operand as a plain 2D
tile of the [pixels, channels] activation matrix instead of through TMA
im2col.  Each case checks that the launch took that path (ie_cuda_last_plan)
and the result: bit-exact with the int8 oracle, max |err| <= 1e-3 * max |ref|
for fp32 (bf16x3).  Pixel counts that are not a multiple of the tile rows put
the zero-filled tail rows to work; channel counts below the 32-byte K step,
one sub-tile or two, and 64..512 output channels cover the tile shapes."""
import numpy as np
import pytest

from tests.qconv import make_q8_problem, run_conv_q8_gpu

pytestmark = pytest.mark.gpu

# (n, c, h, w, m)
Q8_CASES = [
    (3, 64, 11, 11, 256),    # 363 pixels: a partial last tile
    (1, 128, 7, 7, 512),     # 49 pixels: one partial tile
    (2, 256, 14, 14, 64),    # 64 output channels
    (1, 32, 9, 13, 96),      # 32-byte channel blocks, partial output-channel tile
    (2, 48, 5, 5, 16),       # 48 stored channels, K padded to the 32-byte step
    (4, 512, 7, 7, 2048),    # stage-4 expansion shape
]


@pytest.mark.parametrize("case", Q8_CASES, ids=lambda c: "x".join(map(str, c)))
def test_tiled_a_int8_bit_exact(oracle, case):
    from computeengine_b200 import _lib as L
    n, c, h, w, m = case
    rng = np.random.default_rng(n * 7 + c + m)
    x, wq, bias, mult = make_q8_problem(rng, n, c, h, w, m, 1, 1, s_y=0.05 * np.sqrt(c) * 3.0)
    got = run_conv_q8_gpu(x, wq, bias, mult)
    assert L.last_plan().a_tiled == 1, "2D tiled A path not selected"
    want = oracle.conv2d_q8(x, wq, bias, mult, 128, 0, 0, 255)
    np.testing.assert_array_equal(got, want)
    assert ((want > 0) & (want < 255)).mean() > 0.2


def test_strided_and_padded_1x1_keep_im2col(oracle):
    from computeengine_b200 import _lib as L
    n, c, h, w, m = 2, 64, 12, 12, 128
    x, wq, bias, mult = make_q8_problem(np.random.default_rng(3), n, c, h, w, m, 1, 1,
                                        s_y=0.05 * np.sqrt(c) * 3.0)
    for stride, pads in (((2, 2), (0, 0, 0, 0)), ((1, 1), (1, 1, 1, 1))):
        got = run_conv_q8_gpu(x, wq, bias, mult, stride=stride, pads=pads)
        assert L.last_plan().a_tiled == 0
        want = oracle.conv2d_q8(x, wq, bias, mult, 128, 0, 0, 255, strides=stride, pads=pads)
        np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("case", [(3, 64, 11, 11, 256), (2, 96, 9, 9, 128)],
                         ids=lambda c: "x".join(map(str, c)))
def test_tiled_a_f32(oracle, case):
    from computeengine_b200 import _lib as L
    from tests.test_conv_f32_gpu import REL_TOL, run_f32
    n, c, h, w, m = case
    rng = np.random.default_rng(c + m)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / c), (m, c, 1, 1)).astype(np.float32)
    b = rng.normal(0, 0.01, m).astype(np.float32)
    got = run_f32(x, wt, b, act=1)
    assert L.last_plan().a_tiled == 1
    want = oracle.conv2d_f32(x, wt, b, act=1, nthreads=8)
    err = np.abs(got - want).max()
    assert err <= REL_TOL * np.abs(want).max(), err
