"""Row-band mode of the int8 implicit GEMM (stride 1, several filter taps,
resident weights): tiles of whole output rows, one input-band load per channel
block, the taps as shifted operand reads.  Each case checks that the launch
took that mode (ie_cuda_last_plan) and that the output is bit-exact with the
int8 oracle.  The cases cover 32-, 64- and 128-byte channel blocks (the three
operand swizzles), several channel blocks, 5x5, 1x3, 3x1, dilation 2,
asymmetric padding and signed / clamped outputs."""
import numpy as np
import pytest

from tests.qconv import make_q8_problem, run_conv_q8_gpu, tile_policy

pytestmark = pytest.mark.gpu

# (n, c, h, w, m, kh, kw, dil, pads)
CASES = [
    (2, 64, 56, 56, 64, 3, 3, 1, (1, 1, 1, 1)),     # 64-byte blocks, the stage-1 3x3
    (2, 128, 28, 28, 64, 3, 3, 1, (1, 1, 1, 1)),    # 128-byte blocks
    (1, 192, 14, 14, 64, 3, 3, 1, (1, 1, 1, 1)),    # three channel blocks
    (2, 32, 30, 30, 64, 3, 3, 1, (1, 1, 1, 1)),     # 32-byte blocks
    (1, 64, 40, 40, 64, 5, 5, 1, (2, 2, 2, 2)),     # 5x5
    (2, 64, 24, 60, 128, 1, 3, 1, (0, 1, 0, 1)),    # 1x3
    (2, 64, 30, 20, 64, 3, 1, 1, (1, 0, 1, 0)),     # 3x1
    (1, 64, 32, 32, 64, 3, 3, 2, (2, 2, 2, 2)),     # dilation 2
    (2, 64, 33, 33, 64, 3, 3, 1, (0, 2, 1, 0)),     # asymmetric pads
]


def _ids(c):
    return f"{c[0]}x{c[1]}x{c[2]}x{c[3]}_m{c[4]}_{c[5]}x{c[6]}_d{c[7]}_p{''.join(map(str, c[8]))}"


def _run(case, seed, s_y_scale=3.0, **q):
    from computeengine_b200 import _lib as L
    n, c, h, w, m, kh, kw, dil, pads = case
    rng = np.random.default_rng(seed)
    x, wq, bias, mult = make_q8_problem(rng, n, c, h, w, m, kh, kw,
                                        s_y=0.05 * np.sqrt(c * kh * kw) * s_y_scale)
    got = run_conv_q8_gpu(x, wq, bias, mult, pads=pads, dil=(dil, dil), **q)
    plan = L.last_plan()
    return x, wq, bias, mult, got, plan


@pytest.mark.parametrize("policy", ["default", "fill"])
@pytest.mark.parametrize("case", CASES, ids=_ids)
def test_row_band_bit_exact(oracle, case, policy):
    """Under the default tiles every case runs the row-band mode; under the
    fill-the-GPU policy these small launches take 128-position tiles (row band
    or im2col, as the plan estimate decides) and give the same bytes."""
    from computeengine_b200 import _lib as L
    with tile_policy(L.IE_TILE_DEFAULT if policy == "default" else L.IE_TILE_FILL):
        x, wq, bias, mult, got, plan = _run(case, 31 + case[1] + case[5] * 7)
    if policy == "default":
        assert plan.row_band == 1, "row-band mode not selected"
        assert plan.m_sub == 2 or plan.bn == 256
    n, c, h, w, m, kh, kw, dil, pads = case
    want = oracle.conv2d_q8(x, wq, bias, mult, 128, 0, 0, 255, pads=pads, dilations=(dil, dil))
    np.testing.assert_array_equal(got, want)
    assert (want == 0).any() and ((want > 0) & (want < 255)).mean() > 0.2


@pytest.mark.parametrize("y_signed,zp_y,qmin,qmax", [(True, 0, -128, 127), (False, 10, 10, 200),
                                                      (True, -5, -100, 90)])
def test_row_band_output_modes(oracle, y_signed, zp_y, qmin, qmax):
    from computeengine_b200 import _lib as L
    case = CASES[0]
    # a fine output scale so that both clamps are reached
    with tile_policy(L.IE_TILE_DEFAULT):
        x, wq, bias, mult, got, plan = _run(case, 5, s_y_scale=0.06, y_signed=y_signed,
                                            zp_y=zp_y, qmin=qmin, qmax=qmax)
    assert plan.row_band == 1
    want = oracle.conv2d_q8(x, wq, bias, mult, 128, zp_y, qmin, qmax, y_signed=y_signed,
                            pads=case[8])
    np.testing.assert_array_equal(got, want)
    assert (want == qmin).any() and (want == qmax).any()


def test_raw_accumulators_keep_im2col_mode(oracle):
    """The raw int32 output has no staged store, so it stays on im2col tiles."""
    from computeengine_b200 import _lib as L
    case = CASES[0]
    n, c, h, w, m, kh, kw, dil, pads = case
    x, wq, bias, mult = make_q8_problem(np.random.default_rng(2), 1, c, 20, 20, m, kh, kw)
    got = run_conv_q8_gpu(x, wq, bias, mult, pads=pads, raw_acc=True)
    assert L.last_plan().row_band == 0
    _, acc = oracle.conv2d_q8(x, wq, bias, mult, 128, 0, 0, 255, pads=pads, want_acc=True)
    np.testing.assert_array_equal(got, acc + bias.reshape(1, -1, 1, 1))
