"""8-bit NHWC max pooling on the B200 against numpy, bit-exact: uint8 and
int8 values, the 3x3 / stride-2 windows of the ResNet stem (the row-walking
kernel, pads 0, 1 and 2, output heights that leave a short last chunk) and of
a stride-1 pool, a non-3x3 window (the general loop), odd sizes whose last
windows hang over the bottom and right edges, and a value range that puts the
maximum in the padding corners' reach.  Padding never wins, like the
reference's MaxPool2D (pool_ops.cpp)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def maxpool_nhwc_numpy(x: np.ndarray, k: int, stride: int, pad: int) -> np.ndarray:
    n, h, w, c = x.shape
    oh = (h + 2 * pad - k) // stride + 1
    ow = (w + 2 * pad - k) // stride + 1
    out = np.empty((n, oh, ow, c), x.dtype)
    for oy in range(oh):
        y0, y1 = max(oy * stride - pad, 0), min(oy * stride - pad + k, h)
        for ox in range(ow):
            x0, x1 = max(ox * stride - pad, 0), min(ox * stride - pad + k, w)
            out[:, oy, ox, :] = x[:, y0:y1, x0:x1, :].max(axis=(1, 2))
    return out


CASES = [
    # n, h, w, c_store, k, stride, pad, signed
    (2, 112, 112, 64, 3, 2, 1, False),  # ResNet stem pool
    (2, 112, 112, 64, 3, 2, 1, True),
    (1, 13, 9, 32, 3, 2, 1, True),      # odd sizes: edge windows on both sides
    (2, 7, 11, 16, 3, 1, 1, False),     # stride 1
    (1, 10, 10, 48, 2, 2, 0, True),     # general path (k = 2)
    (1, 9, 7, 16, 5, 2, 2, False),      # general path, wide padding
    (3, 17, 9, 16, 3, 2, 1, False),     # 3x3 / 2 row walk: 9 output rows, a short last chunk
    (1, 15, 15, 32, 3, 2, 0, True),     # 3x3 / 2 without padding
    (2, 10, 12, 16, 3, 2, 2, True),     # 3x3 / 2, pad 2: windows with one in-image row
]


@pytest.mark.parametrize("n,h,w,c,k,stride,pad,signed", CASES)
def test_maxpool_q8_matches_numpy(n, h, w, c, k, stride, pad, signed):
    import torch
    from computeengine_b200 import _lib as L

    rng = np.random.default_rng(h * 100 + w + c + k)
    if signed:
        x = rng.integers(-128, 128, (n, h, w, c), dtype=np.int8)
        # all-negative windows: a zero from the padding would win if it took part
        x[:, :3, :3, :] = -120
    else:
        x = rng.integers(0, 256, (n, h, w, c), dtype=np.uint8)
    want = maxpool_nhwc_numpy(x, k, stride, pad)
    xd = torch.from_numpy(x.view(np.uint8)).cuda()
    yd = torch.full(want.shape, 0x5A, dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_q8_maxpool2d(xd.data_ptr(), yd.data_ptr(), n, h, w, c, k, stride, pad,
                                       1 if signed else 0, None))
    torch.cuda.synchronize()
    got = yd.cpu().numpy().view(x.dtype)
    np.testing.assert_array_equal(got, want)
