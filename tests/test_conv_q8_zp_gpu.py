"""Any activation zero point on the dense int8 tensor-core path, bit-exact
with the int8 oracle.

The scheme's activations are per-tensor asymmetric (uint8 or int8 with any
zero point), and the padding of a quantized convolution is real 0.0, i.e.
the stored value zp_x.  The kernel reads a haloed input whose border holds
zp_x (ie_cuda_q8_pack_input_halo) and folds -zp_x * sum(w) into the bias,
so each tap contributes (x - zp_x) * w.  The cases cover the im2col (1x1,
3x3 pad 1, 3x3 stride 2, 7x7 stride 2), tiled-A and row-band modes, raw
accumulators and requantized outputs, uint8 and int8 activations."""
import numpy as np
import pytest

from tests.qconv import make_q8_problem, run_conv_q8_gpu

pytestmark = pytest.mark.gpu

ZPS = [1, 37, 127, 129, 200, 255]

# (n, c, h, w, m, kh, kw, stride, pads, mode)
SHAPES = [
    (2, 64, 14, 14, 64, 1, 1, (1, 1), (0, 0, 0, 0), "tiled"),
    (2, 64, 15, 13, 96, 3, 3, (1, 1), (1, 1, 1, 1), "any"),
    (2, 64, 15, 13, 64, 3, 3, (2, 2), (1, 1, 1, 1), "im2col"),
    (1, 3, 30, 30, 64, 7, 7, (2, 2), (3, 3, 3, 3), "im2col"),
    (2, 64, 56, 56, 64, 3, 3, (1, 1), (1, 1, 1, 1), "rowband"),
    (1, 32, 9, 11, 16, 3, 3, (1, 1), (0, 2, 1, 0), "any"),
]


def _ids(c):
    return f"{c[0]}x{c[1]}x{c[2]}x{c[3]}_m{c[4]}_{c[5]}x{c[6]}_s{c[7][0]}_{c[9]}"


def _check_mode(mode):
    from computeengine_b200 import _lib as L
    plan = L.last_plan()
    if mode == "tiled":
        assert plan.a_tiled == 1
    elif mode == "rowband":
        assert plan.row_band == 1
    elif mode == "im2col":
        assert plan.row_band == 0 and plan.a_tiled == 0


@pytest.mark.parametrize("shape", SHAPES, ids=_ids)
@pytest.mark.parametrize("zp", ZPS)
def test_uint8_zero_point_requantized(oracle, shape, zp):
    n, c, h, w, m, kh, kw, stride, pads, mode = shape
    rng = np.random.default_rng(1000 * zp + c + kh)
    x, wq, bias, mult = make_q8_problem(rng, n, c, h, w, m, kh, kw, x_zp=zp, x_std=45.0,
                                        s_y=0.05 * np.sqrt(c * kh * kw) * 2.5)
    got = run_conv_q8_gpu(x, wq, bias, mult, stride=stride, pads=pads, zp_x=zp)
    want = oracle.conv2d_q8(x, wq, bias, mult, zp, 0, 0, 255, strides=stride, pads=pads)
    np.testing.assert_array_equal(got, want)
    assert 0.05 < np.mean((want > 0) & (want < 255)), "problem should not be all-saturated"
    _check_mode(mode)


@pytest.mark.parametrize("shape", [s for s in SHAPES if s[9] != "rowband"], ids=_ids)
@pytest.mark.parametrize("zp", [1, 129, 255])
def test_uint8_zero_point_accumulators(oracle, shape, zp):
    n, c, h, w, m, kh, kw, stride, pads, mode = shape
    rng = np.random.default_rng(77 * zp + m)
    x, wq, bias, mult = make_q8_problem(rng, n, c, h, w, m, kh, kw, x_zp=zp, x_std=60.0)
    got = run_conv_q8_gpu(x, wq, bias, mult, stride=stride, pads=pads, zp_x=zp, raw_acc=True)
    _, acc = oracle.conv2d_q8(x, wq, bias, mult, zp, 0, 0, 255, want_acc=True, strides=stride,
                              pads=pads)
    np.testing.assert_array_equal(got, acc + bias.reshape(1, -1, 1, 1))


@pytest.mark.parametrize("zp", [-128, -50, 77, 127])
def test_int8_zero_point_signed_output(oracle, zp):
    """int8 activations with a nonzero zero point, int8 output with its own
    zero point and clamp (sign-corrected requantize)."""
    rng = np.random.default_rng(500 + zp)
    n, c, h, w, m = 2, 48, 12, 10, 80
    x = np.clip(np.rint(rng.normal(zp, 40, (n, c, h, w))), -128, 127).astype(np.int8)
    _, wq, bias, mult = make_q8_problem(rng, 1, c, 1, 1, m, 3, 3, s_y=0.05 * np.sqrt(c * 9) * 2)
    got = run_conv_q8_gpu(x, wq, bias, mult, pads=(1, 1, 1, 1), zp_x=zp, zp_y=-7, qmin=-100,
                          qmax=110, y_signed=True)
    want = oracle.conv2d_q8(x, wq, bias, mult, zp, -7, -100, 110, y_signed=True,
                            pads=(1, 1, 1, 1))
    np.testing.assert_array_equal(got, want)


def test_zero_point_128_halo_equals_xor_rebasing(oracle):
    """uint8 zero point 128 through the haloed input gives the same bytes as
    the XOR re-basing to int8 with zero point 0."""
    rng = np.random.default_rng(3)
    x, wq, bias, mult = make_q8_problem(rng, 2, 64, 20, 20, 128, 3, 3, s_y=0.05 * 24 * 3)
    a = run_conv_q8_gpu(x, wq, bias, mult, pads=(1, 1, 1, 1))
    b = run_conv_q8_gpu(x, wq, bias, mult, pads=(1, 1, 1, 1), force_halo=True)
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(a, oracle.conv2d_q8(x, wq, bias, mult, 128, 0, 0, 255,
                                                      pads=(1, 1, 1, 1)))


def test_halo_from_nhwc_matches_halo_from_nchw():
    """ie_cuda_q8_halo_nhwc (a previous layer's NHWC output -> haloed input)
    writes the same bytes as packing the NCHW tensor with its halo."""
    import torch
    from computeengine_b200 import _lib as L
    from tests.qconv import desc_for
    rng = np.random.default_rng(8)
    n, c, h, w = 2, 40, 9, 13
    x = rng.integers(0, 256, (n, c, h, w), dtype=np.uint8)
    d = desc_for(L, n, c, h, w, 16, 3, 5, (1, 2), (1, 2, 2, 0))
    st = torch.cuda.current_stream().cuda_stream
    cs = 48
    xd = torch.from_numpy(x).cuda()
    plain = torch.zeros((n, h, w, cs), dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_q8_pack_input(xd.data_ptr(), plain.data_ptr(), n, c, h, w, cs, 0, st))
    hb = int(L.lib.ie_cuda_q8_halo_input_bytes(d))
    a = torch.zeros(hb, dtype=torch.uint8, device="cuda")
    b = torch.zeros(hb, dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_q8_pack_input_halo(d, xd.data_ptr(), a.data_ptr(), 201, st))
    L.check(L.lib.ie_cuda_q8_halo_nhwc(d, plain.data_ptr(), b.data_ptr(), 201, st))
    torch.cuda.synchronize()
    ha = a.cpu().numpy().reshape(n, h + 3, w + 2, cs)
    hbn = b.cpu().numpy().reshape(n, h + 3, w + 2, cs)
    np.testing.assert_array_equal(ha[..., :c], hbn[..., :c])
    np.testing.assert_array_equal(ha[:, 1:1 + h, 2:2 + w, :c], x.transpose(0, 2, 3, 1))
    assert (ha[:, 0] == 201).all() and (ha[:, :, :2] == 201).all() and (ha[:, -2:] == 201).all()
