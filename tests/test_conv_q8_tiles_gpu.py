"""Tile choice of the int8 implicit GEMM (ie_cuda_set_tile_policy).  A launch
whose default tiles (256 positions below 256 channels) cannot fill the 148
SMs takes narrower or shorter tiles under the default IE_TILE_FILL policy:
128-position tiles of 64 or 128 channels, in row-band, im2col or 2D-tiled
mode, with resident or streamed weights.  Each case checks which plan ran
(ie_cuda_last_plan) under both policies and that both give the oracle's
bytes."""
import numpy as np
import pytest

from tests.qconv import make_q8_problem, run_conv_q8_gpu, tile_policy

pytestmark = pytest.mark.gpu

# (n, c, h, w, m, kh, kw, stride, pads, zp_x, y_signed)
CASES = [
    (8, 128, 28, 28, 128, 3, 3, (1, 1), (1, 1, 1, 1), 128, False),  # the single-conv workload
    (64, 960, 7, 7, 160, 1, 1, (1, 1), (0, 0, 0, 0), 128, False),   # MobileNetV2 b14 projection
    (64, 384, 14, 14, 96, 1, 1, (1, 1), (0, 0, 0, 0), 128, False),  # MobileNetV2 b10 projection
    (4, 64, 14, 14, 64, 3, 3, (1, 1), (1, 1, 1, 1), 37, False),     # haloed input, zero point 37
    (3, 96, 15, 13, 64, 3, 3, (2, 2), (1, 1, 1, 1), 128, True),     # stride 2, int8 output
    (2, 256, 9, 9, 512, 3, 3, (1, 1), (1, 1, 1, 1), 128, False),    # deep K, streamed weights
]


def _ids(c):
    return f"{c[0]}x{c[1]}x{c[2]}x{c[3]}_m{c[4]}_{c[5]}x{c[6]}_s{c[7][0]}_zp{c[9]}{'_s8' if c[10] else ''}"


def _run(oracle, case, policy):
    from computeengine_b200 import _lib as L
    n, c, h, w, m, kh, kw, stride, pads, zp, y_signed = case
    rng = np.random.default_rng(7 + c + m + kh)
    x, wq, bias, mult = make_q8_problem(rng, n, c, h, w, m, kh, kw, x_zp=zp,
                                        s_y=0.05 * np.sqrt(c * kh * kw) * 2.5)
    qmin, qmax = (-128, 127) if y_signed else (0, 255)
    with tile_policy(policy):
        got = run_conv_q8_gpu(x, wq, bias, mult, stride=stride, pads=pads, zp_x=zp,
                              y_signed=y_signed, qmin=qmin, qmax=qmax)
        plan = L.last_plan()
    want = oracle.conv2d_q8(x, wq, bias, mult, zp, 0, qmin, qmax, y_signed=y_signed,
                            strides=stride, pads=pads, nthreads=8)
    np.testing.assert_array_equal(got, want)
    assert ((want > qmin) & (want < qmax)).mean() > 0.05
    return plan


@pytest.mark.parametrize("case", CASES, ids=_ids)
def test_fill_policy_bit_exact(oracle, case):
    from computeengine_b200 import _lib as L
    fill = _run(oracle, case, L.IE_TILE_FILL)
    default = _run(oracle, case, L.IE_TILE_DEFAULT)
    assert default.m_sub == 2 or default.bn == 256
    # the default plan under-fills every case: the fill policy launches more CTAs
    assert default.grid < 148
    assert fill.grid > default.grid
    assert fill.m_sub == 1 or fill.bn < default.bn


def test_single_conv_workload_plan(oracle):
    """[8,128,28,28] 3x3 -> 128: 25-32 CTAs of 256x128 tiles by default; the
    fill policy runs 128-position x 64-channel row-band tiles on 112 CTAs."""
    from computeengine_b200 import _lib as L
    plan = _run(oracle, CASES[0], L.IE_TILE_FILL)
    assert (plan.bn, plan.m_sub, plan.row_band) == (64, 1, 1)
    assert plan.grid == 112


def test_full_launch_keeps_default_tiles(oracle):
    """A launch that fills the GPU with the default tiles keeps them."""
    from computeengine_b200 import _lib as L
    case = (32, 64, 56, 56, 64, 1, 1, (1, 1), (0, 0, 0, 0), 128, False)
    plan = _run(oracle, case, L.IE_TILE_FILL)
    assert (plan.bn, plan.m_sub) == (64, 2) and plan.grid == 148



@pytest.mark.parametrize("case", [
    (4, 32, 56, 56, 16, 1, 1, (1, 1), (0, 0, 0, 0), 128, False),  # MobileNetV2 b00 projection shape
    (2, 64, 30, 30, 24, 3, 3, (1, 1), (1, 1, 1, 1), 128, False),  # row band, 24 channels
    (3, 96, 15, 13, 32, 3, 3, (2, 2), (1, 1, 1, 1), 37, True),    # stride 2, haloed input, int8 output
], ids=_ids)
def test_narrow_layers_run_32_channel_tiles(oracle, case):
    """int8 layers of at most 32 output channels run 32-channel tiles (two
    128-position sub-tiles, 32-byte staging panels with the 32-byte TMA
    swizzle) instead of 64-channel tiles that are half padding; bit-exact."""
    from computeengine_b200 import _lib as L
    plan = _run(oracle, case, L.IE_TILE_DEFAULT)
    assert (plan.bn, plan.m_sub) == (32, 2)
    fill = _run(oracle, case, L.IE_TILE_FILL)
    assert fill.bn == 32
