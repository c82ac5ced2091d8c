"""Depthwise int8 convolution (CUDA cores, NHWC, 128-bit channel vectors)
against the int8 oracle run as a grouped convolution with group == C
(the reference's DepthwiseConv2DOp semantics, conv2d_op.h:53-67).
Bit-exact, including any input zero point (padding is real 0)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def run_dw_gpu(x, w, bias, mult, *, stride, pad, zp_x, zp_y, qmin, qmax, y_signed=False,
               pads=None):
    import torch
    from computeengine_b200 import _lib as L
    from tests.qconv import desc_for
    n, c, h, ww = x.shape
    k = w.shape[2]
    d = desc_for(L, n, c, h, ww, c, k, k, (stride, stride), pads or (pad,) * 4, (1, 1), c, 0, 1)
    s = L.ConvShape()
    L.check(L.lib.ie_conv2d_resolve(d, c, s))
    cs = (c + 15) // 16 * 16
    stream = torch.cuda.current_stream().cuda_stream
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    x_nhwc = torch.zeros((n, h, ww, cs), dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_q8_pack_input(xd.data_ptr(), x_nhwc.data_ptr(), n, c, h, ww, cs, 0, stream))
    packed = torch.zeros(int(L.lib.ie_cuda_dw_q8_packed_weight_bytes(d)), dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_dw_q8_pack_weights(d, torch.from_numpy(w).cuda().data_ptr(),
                                             packed.data_ptr(), stream))
    q = L.Q8Params()
    q.x_signed, q.zp_x, q.y_signed, q.zp_y, q.qmin, q.qmax = int(x.dtype == np.int8), zp_x, \
        int(y_signed), zp_y, qmin, qmax
    y = torch.full((n, s.out_h, s.out_w, cs), 99, dtype=torch.uint8, device="cuda")
    bd, md = torch.from_numpy(bias).cuda(), torch.from_numpy(mult).cuda()
    L.check(L.lib.ie_cuda_dwconv2d_q8(d, q, x_nhwc.data_ptr(), packed.data_ptr(), bd.data_ptr(),
                                      md.data_ptr(), y.data_ptr(), stream))
    torch.cuda.synchronize()
    assert L.take_device_error() == 0
    out = y[..., :c].permute(0, 3, 1, 2).contiguous().cpu().numpy()
    return out.view(np.int8) if y_signed else out


CASES = [
    # (n, c, h, w, k, stride, pad, zp_x, signed_in)
    (2, 32, 16, 16, 3, 1, 1, 128, False),
    (2, 96, 15, 13, 3, 2, 1, 0, False),
    (1, 144, 14, 14, 3, 1, 1, 0, False),
    (1, 24, 9, 9, 3, 2, 1, 7, False),        # c not a multiple of 16, odd zero point
    (3, 48, 8, 8, 5, 1, 2, 0, True),         # int8 input, 5x5
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(map(str, c[:6])))
def test_depthwise_bit_exact(oracle, case):
    n, c, h, w, k, stride, pad, zp_x, signed_in = case
    rng = np.random.default_rng(c * 7 + k)
    if signed_in:
        x = rng.integers(-100, 101, (n, c, h, w)).astype(np.int8)
    else:
        x = np.clip(np.rint(rng.normal(zp_x + 40, 40, (n, c, h, w))), 0, 255).astype(np.uint8)
    wq = rng.integers(-127, 128, (c, 1, k, k)).astype(np.int8)
    bias = rng.integers(-2000, 2000, c).astype(np.int32)
    mult = rng.uniform(0.001, 0.01, c).astype(np.float32)
    zp_y, qmin, qmax = 0, 0, 120  # ReLU6 at output scale 0.05
    got = run_dw_gpu(x, wq, bias, mult, stride=stride, pad=pad, zp_x=zp_x, zp_y=zp_y, qmin=qmin,
                     qmax=qmax)
    want = oracle.conv2d_q8(x, wq, bias, mult, zp_x, zp_y, qmin, qmax, strides=(stride, stride),
                            pads=(pad,) * 4, group=c, depthwise=True)
    np.testing.assert_array_equal(got, want)
    assert (want == qmax).any() and (want == qmin).any()


def test_depthwise_signed_output_general_zero_point(oracle):
    rng = np.random.default_rng(3)
    x = rng.integers(0, 256, (2, 64, 12, 12)).astype(np.uint8)
    wq = rng.integers(-127, 128, (64, 1, 3, 3)).astype(np.int8)
    bias = rng.integers(-2000, 2000, 64).astype(np.int32)
    mult = rng.uniform(0.0005, 0.004, 64).astype(np.float32)
    got = run_dw_gpu(x, wq, bias, mult, stride=1, pad=1, zp_x=100, zp_y=-3, qmin=-128, qmax=127,
                     y_signed=True)
    want = oracle.conv2d_q8(x, wq, bias, mult, 100, -3, -128, 127, y_signed=True, pads=(1,) * 4,
                            group=64, depthwise=True)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("mult_range,zp_y,qmin,qmax,y_signed", [
    ((0.25, 0.9), 0, 0, 255, False),       # shifts <= 32: exact per-column requantize
    ((0.001, 0.01), 0, -128, 127, True),    # zp_y > qmin: sign-corrected rounding
    ((0.001, 0.01), 3, 3, 100, False),      # folded addend with a narrower clamp
    ((0.001, 0.01), 0, 0, 255, False),      # folded addend, the saturating pack alone clamps
])
def test_depthwise_requantize_modes(oracle, mult_range, zp_y, qmin, qmax, y_signed):
    rng = np.random.default_rng(17)
    c = 80
    x = rng.integers(0, 256, (2, c, 17, 19)).astype(np.uint8)
    wq = rng.integers(-127, 128, (c, 1, 3, 3)).astype(np.int8)
    bias = rng.integers(-3000, 3000, c).astype(np.int32)
    mult = rng.uniform(*mult_range, c).astype(np.float32)
    mult[::7] = 0.125  # exact .5 ties
    scale = 0.02 if mult_range[0] >= 0.25 else 1.0
    mult = (mult * scale).astype(np.float32)
    got = run_dw_gpu(x, wq, bias, mult, stride=1, pad=1, zp_x=20, zp_y=zp_y, qmin=qmin, qmax=qmax,
                     y_signed=y_signed)
    want = oracle.conv2d_q8(x, wq, bias, mult, 20, zp_y, qmin, qmax, y_signed=y_signed,
                            pads=(1,) * 4, group=c, depthwise=True)
    np.testing.assert_array_equal(got, want)
    assert (want == qmin).any() and (want == qmax).any()


def test_depthwise_zero_point_outside_input_type(oracle):
    """A zero point no uint8 value can hold takes the general per-pixel kernel."""
    rng = np.random.default_rng(4)
    c = 48
    x = rng.integers(0, 256, (1, c, 10, 12)).astype(np.uint8)
    wq = rng.integers(-127, 128, (c, 1, 3, 3)).astype(np.int8)
    bias = rng.integers(-2000, 2000, c).astype(np.int32)
    mult = rng.uniform(0.0005, 0.002, c).astype(np.float32)
    got = run_dw_gpu(x, wq, bias, mult, stride=2, pad=1, zp_x=-20, zp_y=0, qmin=0, qmax=255)
    want = oracle.conv2d_q8(x, wq, bias, mult, -20, 0, 0, 255, strides=(2, 2), pads=(1,) * 4,
                            group=c, depthwise=True)
    np.testing.assert_array_equal(got, want)


def test_depthwise_wide_rows_5x5_stride2(oracle):
    """Several 4-pixel steps per row, a ragged last step, 5x5 stride 2."""
    rng = np.random.default_rng(8)
    c = 112
    x = rng.integers(-128, 128, (2, c, 31, 45)).astype(np.int8)
    wq = rng.integers(-127, 128, (c, 1, 5, 5)).astype(np.int8)
    bias = rng.integers(-2000, 2000, c).astype(np.int32)
    mult = rng.uniform(0.0005, 0.004, c).astype(np.float32)
    got = run_dw_gpu(x, wq, bias, mult, stride=2, pad=2, zp_x=-7, zp_y=0, qmin=0, qmax=120)
    want = oracle.conv2d_q8(x, wq, bias, mult, -7, 0, 0, 120, strides=(2, 2), pads=(2,) * 4,
                            group=c, depthwise=True)
    np.testing.assert_array_equal(got, want)
    assert (want == 0).any() and (want == 120).any()


@pytest.mark.parametrize("stride,pads,signed_in,zp_x", [
    (1, (0, 1, 1, 0), False, 255),   # asymmetric pads, zero point at the top of uint8
    (2, (1, 0, 0, 1), True, -128),   # stride 2, int8 input at its lowest zero point
    (2, (0, 0, 0, 0), False, 0),     # no padding, ragged column groups
    (1, (1, 1, 1, 1), True, 33),
])
def test_depthwise_3x3_row_kernel_edges(oracle, stride, pads, signed_in, zp_x):
    """The 3x3 row kernel (4 channels x 4 columns x 4 rows per thread): image
    sizes that leave partial column groups and row strips, asymmetric pads and
    extreme zero points (padding reads as the zero point's byte)."""
    rng = np.random.default_rng(400 + stride + zp_x)
    n, c, h, w = 3, 40, 13, 18
    if signed_in:
        x = rng.integers(-128, 128, (n, c, h, w)).astype(np.int8)
    else:
        x = rng.integers(0, 256, (n, c, h, w)).astype(np.uint8)
    wq = rng.integers(-127, 128, (c, 1, 3, 3)).astype(np.int8)
    bias = rng.integers(-3000, 3000, c).astype(np.int32)
    mult = rng.uniform(0.0008, 0.004, c).astype(np.float32)
    got = run_dw_gpu(x, wq, bias, mult, stride=stride, pad=0, pads=pads, zp_x=zp_x, zp_y=4,
                     qmin=4, qmax=200)
    want = oracle.conv2d_q8(x, wq, bias, mult, zp_x, 4, 4, 200, strides=(stride, stride),
                            pads=pads, group=c, depthwise=True)
    np.testing.assert_array_equal(got, want)
    assert (want == 4).any() and (want == 200).any()
