"""int8 implicit-GEMM convolution (tcgen05 kind::i8) against the int8 oracle,
through the C ABI.  Bit-exact: integer accumulators, then the requantize rule
(round half away from zero, saturate) on identical fp32 multipliers."""
import numpy as np
import pytest

from tests.qconv import make_q8_problem, run_conv_q8_gpu

pytestmark = pytest.mark.gpu

# (n, c, h, w, m, kh, kw, stride, pads)
ACC_CASES = [
    (1, 64, 16, 16, 64, 1, 1, (1, 1), (0, 0, 0, 0)),      # plain GEMM, 2 M tiles
    (1, 64, 16, 16, 64, 3, 3, (1, 1), (1, 1, 1, 1)),      # 3x3 pad 1
    (2, 128, 14, 14, 128, 3, 3, (1, 1), (1, 1, 1, 1)),    # tile crosses images
    (1, 256, 7, 7, 256, 1, 1, (1, 1), (0, 0, 0, 0)),      # BN 256, tail tile
    (2, 64, 15, 13, 96, 3, 3, (2, 2), (1, 1, 1, 1)),      # stride 2, odd sizes
    (1, 48, 12, 12, 32, 1, 1, (2, 2), (0, 0, 0, 0)),      # 1x1 stride 2, c not /64
    (1, 16, 20, 20, 64, 7, 7, (2, 2), (3, 3, 3, 3)),      # 7x7 stride 2
    (3, 512, 7, 7, 512, 3, 3, (1, 1), (1, 1, 1, 1)),      # deep K
    (1, 32, 9, 11, 16, 3, 3, (1, 1), (0, 2, 1, 0)),       # asymmetric pads, m=16
    (1, 160, 10, 10, 320, 1, 1, (1, 1), (0, 0, 0, 0)),    # c = 160 (32-byte blocks)
]


@pytest.mark.parametrize("case", ACC_CASES, ids=lambda c: "x".join(map(str, c[:7])) + f"_s{c[7][0]}")
def test_accumulators_match_oracle(oracle, case):
    n, c, h, w, m, kh, kw, stride, pads = case
    rng = np.random.default_rng(1234 + n * c + m)
    x, wq, bias, mult = make_q8_problem(rng, n, c, h, w, m, kh, kw)
    got = run_conv_q8_gpu(x, wq, bias, mult, stride=stride, pads=pads, raw_acc=True)
    _, acc = oracle.conv2d_q8(x, wq, bias, mult, 128, 0, 0, 255, want_acc=True,
                              strides=stride, pads=pads)
    want = acc + bias.reshape(1, -1, 1, 1)
    assert got.shape == want.shape
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("case", ACC_CASES[:6], ids=lambda c: "x".join(map(str, c[:7])))
def test_requantized_output_bit_exact(oracle, case):
    n, c, h, w, m, kh, kw, stride, pads = case
    rng = np.random.default_rng(99 + c)
    # Output scale chosen so results spread over 0..255 instead of saturating.
    x, wq, bias, mult = make_q8_problem(rng, n, c, h, w, m, kh, kw, s_y=0.05 * np.sqrt(c * kh * kw) * 3)
    got = run_conv_q8_gpu(x, wq, bias, mult, stride=stride, pads=pads)
    want = oracle.conv2d_q8(x, wq, bias, mult, 128, 0, 0, 255, strides=stride, pads=pads)
    np.testing.assert_array_equal(got, want)
    assert 0.05 < np.mean((want > 0) & (want < 255)), "problem should not be all-saturated"


def test_config2_int8_conv_bit_exact(oracle):
    """The single int8 conv workload: x uint8 [8,128,28,28] zp 128 s 0.02,
    w [128,128,3,3] U{-127..127}, s_w U(0.001,0.01), bias N(0,500),
    y uint8 s 0.05 zp 0 with ReLU folded, stride 1 pad 1."""
    rng = np.random.default_rng(0)
    x, wq, bias, mult = make_q8_problem(rng, 8, 128, 28, 28, 128, 3, 3)
    got = run_conv_q8_gpu(x, wq, bias, mult, pads=(1, 1, 1, 1))
    want = oracle.conv2d_q8(x, wq, bias, mult, 128, 0, 0, 255, pads=(1, 1, 1, 1), nthreads=8)
    np.testing.assert_array_equal(got, want)


def test_relu6_clamp_and_unsigned_input(oracle):
    rng = np.random.default_rng(5)
    x, wq, bias, mult = make_q8_problem(rng, 2, 64, 10, 10, 64, 3, 3, x_zp=0, x_std=40,
                                        s_y=0.1)
    zp_y, qmax = 3, 3 + 120
    got = run_conv_q8_gpu(x, wq, bias, mult, pads=(1, 1, 1, 1), zp_x=0, zp_y=zp_y, qmin=zp_y,
                          qmax=qmax)
    want = oracle.conv2d_q8(x, wq, bias, mult, 0, zp_y, zp_y, qmax, pads=(1, 1, 1, 1))
    np.testing.assert_array_equal(got, want)
    assert want.min() == zp_y and want.max() == qmax


def _run_1x1_signed_input(x, wq, bias, mult, y_signed, zp_y, qmin, qmax):
    """int8 NHWC input, 1x1 convolution, requantized output as NCHW numpy."""
    import torch
    from computeengine_b200 import _lib as L
    from tests.qconv import desc_for
    n, c, h, w = x.shape
    m = wq.shape[0]
    d = desc_for(L, n, c, h, w, m, 1, 1)
    stream = torch.cuda.current_stream().cuda_stream
    x_nhwc = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 3, 1))).cuda()
    packed = torch.zeros(int(L.lib.ie_cuda_q8_packed_weight_bytes(d)), dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_q8_pack_weights(d, torch.from_numpy(wq).cuda().data_ptr(), packed.data_ptr(), stream))
    q = L.Q8Params()
    q.x_signed, q.zp_x, q.y_signed, q.zp_y, q.qmin, q.qmax = 1, 0, int(y_signed), zp_y, qmin, qmax
    y = torch.zeros((n, h, w, m), dtype=torch.uint8, device="cuda")
    bd, md = torch.from_numpy(bias).cuda(), torch.from_numpy(mult).cuda()
    L.check(L.lib.ie_cuda_conv2d_q8(d, q, x_nhwc.data_ptr(), packed.data_ptr(), bd.data_ptr(),
                                    md.data_ptr(), y.data_ptr(), stream))
    torch.cuda.synchronize()
    assert L.take_device_error() == 0
    return y.cpu().numpy().view(np.int8 if y_signed else np.uint8).transpose(0, 3, 1, 2)


def _tie_fraction(acc, bias, mult):
    v = (acc.astype(np.float64) + bias.reshape(1, -1, 1, 1)) * mult.astype(np.float64).reshape(1, -1, 1, 1)
    return np.mean(np.abs(v - np.trunc(v)) == 0.5)


@pytest.mark.parametrize("y_signed,zp_y,qmin,qmax", [(False, 0, 0, 255), (True, 0, -128, 127),
                                                      (False, 10, 10, 200), (True, -5, -100, 90)])
def test_requantize_ties_and_saturation(oracle, y_signed, zp_y, qmin, qmax):
    """Multipliers 2^-k and 3*2^-k make many requantized values exact .5 ties
    (round half away from zero), others saturate.  Multipliers of 0.25 and
    above put every warp on the epilogue's exact per-column path."""
    rng = np.random.default_rng(11)
    n, c, h, w, m = 2, 32, 9, 9, 64
    x = rng.integers(-60, 61, (n, c, h, w)).astype(np.int8)
    wq = rng.integers(-127, 128, (m, c, 1, 1)).astype(np.int8)
    bias = rng.integers(-3000, 3000, m).astype(np.int32)
    cands = [0.5, 0.25, 0.125, 1.5, 0.75, 0.375, 2.0 ** -10, 3 * 2.0 ** -9, 0.0009765625, 0.01]
    mult = np.array([cands[i % len(cands)] for i in range(m)], np.float32)
    got = _run_1x1_signed_input(x, wq, bias, mult, y_signed, zp_y, qmin, qmax)
    want, acc = oracle.conv2d_q8(x, wq, bias, mult, 0, zp_y, qmin, qmax, y_signed=y_signed,
                                 want_acc=True)
    np.testing.assert_array_equal(got, want)
    assert _tie_fraction(acc, bias, mult) > 0.05
    assert (want == qmin).any() and (want == qmax).any()


# (y_signed, zp_y, qmin, qmax): the output formats and clamp ranges that select
# each fast requantize mode (bias folded into a 64-bit addend when zp_y <= qmin,
# sign-corrected rounding otherwise; saturating pack alone when the clamp range
# is the storage type's)
FAST_MODE_CASES = [
    (False, 0, 0, 255),      # folded addend, no extra clamp
    (False, 10, 10, 200),    # folded addend, clamp
    (True, -128, -128, 127),  # folded addend, int8 output
    (True, 0, -128, 127),    # sign-corrected, no extra clamp
    (True, -5, -100, 90),    # sign-corrected, clamp
    (False, 20, 0, 255),     # sign-corrected, uint8 output
]


@pytest.mark.parametrize("y_signed,zp_y,qmin,qmax", FAST_MODE_CASES)
def test_requantize_fast_modes_ties(oracle, y_signed, zp_y, qmin, qmax):
    """Multipliers below 0.25 whose shifts lie within 7 of each other keep every
    warp on a fast mode; small operands and multipliers such as 1/8 and 1/16
    make many products exact .5 ties of either sign."""
    rng = np.random.default_rng(23)
    n, c, h, w, m = 2, 32, 11, 9, 192
    x = rng.integers(-12, 13, (n, c, h, w)).astype(np.int8)
    wq = rng.integers(-12, 13, (m, c, 1, 1)).astype(np.int8)
    bias = rng.integers(-1500, 1500, m).astype(np.int32)
    cands = [0.125, 0.0625, 0.09375, 2.0 ** -9, 0.1, 0.07, 0.2, 0.015625]
    mult = np.array([cands[i % len(cands)] for i in range(m)], np.float32)
    got = _run_1x1_signed_input(x, wq, bias, mult, y_signed, zp_y, qmin, qmax)
    want, acc = oracle.conv2d_q8(x, wq, bias, mult, 0, zp_y, qmin, qmax, y_signed=y_signed,
                                 want_acc=True)
    np.testing.assert_array_equal(got, want)
    assert _tie_fraction(acc, bias, mult) > 0.02
    assert (want == qmin).any() and (want == qmax).any()
    assert ((want > qmin) & (want < qmax)).mean() > 0.3


def test_requantize_bias_near_int32_limit(oracle):
    """A bias within the accumulator bound of 2^31 cannot be folded into the
    64-bit addend; acc + bias then wraps in int32 exactly as the oracle's does."""
    rng = np.random.default_rng(5)
    n, c, h, w, m = 1, 32, 8, 8, 64
    x = rng.integers(-100, 101, (n, c, h, w)).astype(np.int8)
    wq = rng.integers(-127, 128, (m, c, 1, 1)).astype(np.int8)
    bias = rng.integers(-1000, 1000, m).astype(np.int32)
    bias[::3] = np.int32(2 ** 31 - 1 - 50)
    bias[1::7] = np.int32(-(2 ** 31) + 40)
    mult = np.full(m, 2.0 ** -20, np.float32)
    for y_signed, zp_y, qmin, qmax in ((False, 0, 0, 255), (True, 3, -128, 127)):
        got = _run_1x1_signed_input(x, wq, bias, mult, y_signed, zp_y, qmin, qmax)
        want, acc = oracle.conv2d_q8(x, wq, bias, mult, 0, zp_y, qmin, qmax, y_signed=y_signed,
                                     want_acc=True)
        np.testing.assert_array_equal(got, want)
        t = acc.astype(np.int64) + bias.astype(np.int64).reshape(1, -1, 1, 1)
        assert (t > 2 ** 31 - 1).any() and (t < -(2 ** 31)).any()  # both wraps occur
