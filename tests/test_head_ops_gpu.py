"""The head ops of a ResNet graph on the B200 against the reference's own ops
compiled from its sources (pool_ops.cpp, gemm_op.cpp):

* max / average pooling and global average pooling are bit-exact (same window
  order and arithmetic): the ResNet stem pool, SAME padding, ceil_mode,
  count_include_pad, the 7x7 head average; int8 max pooling on the int8
  activation layout against the same pool on the integers as floats;
* Gemm runs as bf16x3 on the tensor cores: max |err| <= 1e-3 * max |ref|,
  over transA / transB, alpha / beta and every C broadcast, the fused
  column-bias path (the ResNet FC layer 2048 -> 1000) and sizes that are not
  tile multiples."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3
AUTO = {"NOTSET": 0, "VALID": 1, "SAME_UPPER": 2, "SAME_LOWER": 3}

POOLS = [
    # shape, kind, kernel, strides, pads, auto_pad, ceil, count_include_pad
    ((2, 64, 112, 112), "max", (3, 3), (2, 2), (1, 1, 1, 1), "NOTSET", 0, 0),
    ((2, 8, 13, 11), "max", (3, 3), (2, 2), (0, 0, 0, 0), "SAME_UPPER", 0, 0),
    ((2, 8, 13, 11), "avg", (3, 3), (2, 2), (1, 1, 1, 1), "NOTSET", 1, 0),
    ((2, 8, 13, 11), "avg", (3, 3), (1, 1), (1, 1, 1, 1), "NOTSET", 0, 1),
    ((1, 5, 10, 9), "avg", (2, 3), (2, 2), (0, 1, 1, 0), "SAME_LOWER", 0, 0),
    ((4, 2048, 7, 7), "avg", (7, 7), (1, 1), (0, 0, 0, 0), "NOTSET", 0, 0),
]


def _pool_gpu(x, kind, kernel, strides, pads, auto, ceil_mode, cip):
    import torch
    from computeengine_b200 import _lib as L
    d = L.PoolDesc()
    d.n, d.c, d.h, d.w = x.shape
    d.kh, d.kw = kernel
    d.stride_h, d.stride_w = strides
    d.pad_top, d.pad_left, d.pad_bottom, d.pad_right = pads
    d.auto_pad, d.ceil_mode, d.count_include_pad = AUTO[auto], ceil_mode, cip
    s = L.ConvShape()
    L.check(L.lib.ie_pool2d_resolve(d, s))
    xd = torch.from_numpy(x).cuda()
    y = torch.full((x.shape[0], x.shape[1], s.out_h, s.out_w), float("nan"), device="cuda")
    L.check(L.lib.ie_cuda_pool2d_f32(d, 1 if kind == "max" else 0, xd.data_ptr(), y.data_ptr(),
                                     None))
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("case", POOLS, ids=lambda c: f"{c[1]}{c[2][0]}x{c[2][1]}_{c[5]}_c{c[6]}_i{c[7]}")
def test_pool2d_bit_exact(refconv, case):
    shape, kind, kernel, strides, pads, auto, ceil_mode, cip = case
    x = np.random.default_rng(sum(shape)).normal(size=shape).astype(np.float32)
    x[:, :, :2, :2] = -5.0  # negative corners: padding must never win a max
    got = _pool_gpu(x, kind, kernel, strides, pads, auto, ceil_mode, cip)
    rc, want = refconv.pool2d(x, kernel, strides, pads, auto, ceil_mode, cip, kind=kind)
    assert rc == 0
    np.testing.assert_array_equal(got, want)


Q8_POOLS = [
    # shape, kernel, strides, pads, auto_pad, ceil, signed
    ((2, 64, 112, 112), (3, 3), (2, 2), (1, 1, 1, 1), "NOTSET", 0, 0),  # ResNet stem pool
    ((2, 5, 13, 11), (2, 3), (2, 1), (0, 1, 1, 0), "NOTSET", 1, 1),
    ((1, 40, 9, 10), (3, 2), (1, 2), (0, 0, 0, 0), "SAME_LOWER", 0, 0),
    ((1, 24, 8, 8), (3, 3), (3, 3), (0, 0, 0, 0), "SAME_UPPER", 1, 1),
    ((2, 16, 6, 7), (2, 2), (1, 1), (3, 0, 0, 2), "NOTSET", 0, 1),  # windows in the padding only
    ((2, 24, 17, 14), (3, 3), (2, 2), (1, 1, 2, 0), "NOTSET", 0, 1),  # 3x3 / 2 row walk, uneven pads
    ((1, 16, 12, 12), (3, 3), (2, 2), (1, 1, 1, 1), "NOTSET", 1, 0),  # 3x3 / 2 row walk, ceil_mode
    ((1, 16, 9, 9), (3, 3), (2, 2), (1, 1, 3, 3), "NOTSET", 0, 0),    # 3x3 / 2, pads 3: general kernel
]


@pytest.mark.parametrize("case", Q8_POOLS, ids=lambda c: f"c{c[0][1]}_k{c[1][0]}x{c[1][1]}_{c[4]}_c{c[5]}_s{c[6]}")
def test_q8_maxpool_nhwc_bit_exact(refconv, case):
    """int8 max pooling over the int8 activation layout (NHWC, channels padded
    to 16) equals the reference MaxPool2DOp on the same integers as floats;
    a window with no in-image position gives the type's minimum (-inf in
    the reference)."""
    import torch
    from computeengine_b200 import _lib as L
    shape, kernel, strides, pads, auto, ceil_mode, signed = case
    n, c, h, w = shape
    rng = np.random.default_rng(sum(shape) + signed)
    dt = np.int8 if signed else np.uint8
    lo, hi = (-128, 128) if signed else (0, 256)
    x = rng.integers(lo, hi, shape).astype(dt)
    d = L.PoolDesc()
    d.n, d.c, d.h, d.w = shape
    d.kh, d.kw = kernel
    d.stride_h, d.stride_w = strides
    d.pad_top, d.pad_left, d.pad_bottom, d.pad_right = pads
    d.auto_pad, d.ceil_mode, d.count_include_pad = AUTO[auto], ceil_mode, 0
    s = L.ConvShape()
    L.check(L.lib.ie_pool2d_resolve(d, s))
    cs = (c + 15) // 16 * 16
    xn = np.zeros((n, h, w, cs), np.uint8)
    xn[..., :c] = x.view(np.uint8).transpose(0, 2, 3, 1)
    xd = torch.from_numpy(xn).cuda()
    y = torch.full((n, s.out_h, s.out_w, cs), 0x5A, dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_q8_maxpool2d_nhwc(d, signed, xd.data_ptr(), y.data_ptr(), None))
    torch.cuda.synchronize()
    got = y.cpu().numpy()[..., :c].transpose(0, 3, 1, 2).view(dt)
    rc, want = refconv.pool2d(x.astype(np.float32), kernel, strides, pads, auto, ceil_mode, 0,
                              kind="max")
    assert rc == 0
    empty = np.isneginf(want)
    want = np.where(empty, lo, want).astype(dt)
    np.testing.assert_array_equal(got, want)
    if pads[0] >= kernel[0]:
        assert empty.any()


@pytest.mark.parametrize("shape", [(4, 2048, 7, 7), (2, 64, 56, 56), (3, 5, 1, 1)])
def test_global_avg_pool_bit_exact(refconv, shape):
    import torch
    from computeengine_b200 import _lib as L
    x = np.random.default_rng(shape[1]).normal(size=shape).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    y = torch.full((shape[0], shape[1], 1, 1), float("nan"), device="cuda")
    L.check(L.lib.ie_cuda_global_avg_pool_f32(xd.data_ptr(), y.data_ptr(), *shape, None))
    torch.cuda.synchronize()
    rc, want = refconv.pool2d(x, kind="global")
    assert rc == 0
    np.testing.assert_array_equal(y.cpu().numpy(), want)


@pytest.mark.parametrize("shape,signed,zp,scale", [
    ((4, 2048, 7, 7), False, 0, 0.05),   # the ResNet-50 head
    ((2, 40, 7, 7), True, -3, 0.031),    # int8, channels not a multiple of 16
    ((1, 16, 56, 56), False, 131, 0.2),  # a large plane: lanes stride over 3136 pixels
])
def test_q8_global_avg_pool_rule(shape, signed, zp, scale):
    """int8 GlobalAvgPool into fp32: fp32((sum q - zp * hw) * scale / hw), the
    sum exact, the rest in double rounded once -- equal bit for bit."""
    import torch
    from computeengine_b200 import _lib as L
    n, c, h, w = shape
    rng = np.random.default_rng(c + h)
    dt = np.int8 if signed else np.uint8
    lo, hi = (-128, 128) if signed else (0, 256)
    x = rng.integers(lo, hi, shape).astype(dt)
    cs = (c + 15) // 16 * 16
    xn = np.full((n, h, w, cs), 0x7F, np.uint8)
    xn[..., :c] = x.view(np.uint8).transpose(0, 2, 3, 1)
    xd = torch.from_numpy(xn).cuda()
    y = torch.full((n, c), float("nan"), device="cuda")
    L.check(L.lib.ie_cuda_q8_global_avg_pool_nhwc(xd.data_ptr(), y.data_ptr(), n, c, h, w,
                                                   int(signed), zp, scale, None))
    torch.cuda.synchronize()
    hw = h * w
    want = ((x.astype(np.int64).sum(axis=(2, 3)).astype(np.float64) - np.float64(zp) * hw)
            * np.float64(scale) / np.float64(hw)).astype(np.float32)
    np.testing.assert_array_equal(y.cpu().numpy(), want)


C_MODE = {"none": 0, "scalar": 1, "row": 2, "column": 3, "full": 4}

GEMMS = [
    # m, n, k, trans_a, trans_b, alpha, beta, c
    (256, 1000, 2048, 0, 1, 1.0, 1.0, "column"),  # ResNet FC: fused bias
    (37, 50, 70, 0, 0, 1.0, 1.0, "none"),
    (37, 50, 70, 1, 0, 0.5, 2.0, "full"),
    (64, 33, 16, 1, 1, -1.5, 0.25, "row"),
    (130, 129, 200, 0, 1, 2.0, -1.0, "scalar"),
    (5, 7, 3, 0, 0, 1.0, 3.0, "column"),
]


@pytest.mark.parametrize("case", GEMMS, ids=lambda c: f"{c[0]}x{c[1]}x{c[2]}_t{c[3]}{c[4]}_{c[7]}")
def test_gemm_matches_reference(refconv, case):
    import torch
    from computeengine_b200 import _lib as L
    m, n, k, ta, tb, alpha, beta, cm = case
    rng = np.random.default_rng(m + n + k)
    a = rng.normal(size=(k, m) if ta else (m, k)).astype(np.float32)
    b = rng.normal(size=(n, k) if tb else (k, n)).astype(np.float32)
    c = {"none": None, "scalar": rng.normal(size=(1,)), "row": rng.normal(size=(m, 1)),
         "column": rng.normal(size=(n,)), "full": rng.normal(size=(m, n))}[cm]
    c = None if c is None else c.astype(np.float32)
    rc, want = refconv.gemm(a, b, c, alpha, beta, ta, tb)
    assert rc == 0
    ad, bd = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    cd = torch.from_numpy(np.ascontiguousarray(c)).cuda() if c is not None else None
    y = torch.full((m, n), float("nan"), device="cuda")
    nbytes = int(L.lib.ie_cuda_gemm_f32_workspace_bytes(m, n, k, ta, tb))
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_gemm_f32(m, n, k, ta, tb, alpha, beta, ad.data_ptr(), bd.data_ptr(),
                                   cd.data_ptr() if cd is not None else None, C_MODE[cm],
                                   y.data_ptr(), ws.data_ptr(), nbytes, None))
    torch.cuda.synchronize()
    assert L.take_device_error() == 0
    err = np.abs(y.cpu().numpy() - want).max()
    assert err <= REL_TOL * np.abs(want).max(), err
