"""Residual-add fusion of the fp32 convolution: y = act((conv(x, w) + b) + r),
the ResNet bottleneck's add run in the convolution's epilogue.  Against the
oracle's fp32 convolution followed by the add and the activation in fp32:
max |err| <= 1e-3 * max |ref|.  NCHW drop-in (also with the output written in
place over the residual) and the NHWC bf16x3 building block; grouped
convolutions are rejected."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def _problem(n, c, h, w, m, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / (c * k * k)), (m, c, k, k)).astype(np.float32)
    b = rng.normal(0, 0.05, m).astype(np.float32)
    return x, wt, b


@pytest.mark.parametrize("shape,act", [((2, 64, 14, 14, 256, 1), 1), ((1, 32, 9, 11, 48, 3), 0),
                                       ((3, 16, 7, 7, 64, 1), 2)])
@pytest.mark.parametrize("in_place", [False, True])
def test_f32_residual_nchw(oracle, shape, act, in_place):
    import torch
    from computeengine_b200 import _lib as L
    from tests.qconv import desc_for
    n, c, h, w, m, k = shape
    x, wt, b = _problem(n, c, h, w, m, k, seed=m + c)
    p = k // 2
    conv = oracle.conv2d_f32(x, wt, b, pads=(p, p, p, p), nthreads=8)
    r = np.random.default_rng(1).normal(0, 1, conv.shape).astype(np.float32)
    want = conv + r
    if act == 1:
        want = np.maximum(want, np.float32(0))
    elif act == 2:
        want = np.clip(want, np.float32(0), np.float32(6))
    d = desc_for(L, n, c, h, w, m, k, k, pads=(p, p, p, p))
    xd, wd, bd = (torch.from_numpy(t).cuda() for t in (x, wt, b))
    rd = torch.from_numpy(r).cuda()
    y = rd if in_place else torch.full(conv.shape, float("nan"), device="cuda")
    nbytes = int(L.lib.ie_cuda_conv2d_f32_workspace_bytes(d))
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_conv2d_f32_residual(d, act, xd.data_ptr(), wd.data_ptr(), bd.data_ptr(),
                                              rd.data_ptr(), y.data_ptr(), ws.data_ptr(), nbytes,
                                              None))
    torch.cuda.synchronize()
    assert L.take_device_error() == 0
    err = np.abs(y.cpu().numpy() - want).max()
    assert err <= REL_TOL * np.abs(want).max(), err


def test_bf16x3_residual_nhwc(oracle):
    import torch
    from computeengine_b200 import _lib as L
    from tests.qconv import desc_for
    n, c, h, w, m = 2, 64, 12, 10, 128
    x, wt, b = _problem(n, c, h, w, m, 1, seed=5)
    conv = oracle.conv2d_f32(x, wt, b, nthreads=8)              # NCHW
    r = np.random.default_rng(2).normal(0, 1, conv.shape).astype(np.float32)
    want = np.maximum(conv + r, np.float32(0)).transpose(0, 2, 3, 1)  # NHWC
    d = desc_for(L, n, c, h, w, m, 1, 1)
    c_store = (c + 15) // 16 * 16
    xd, wd, bd = (torch.from_numpy(t).cuda() for t in (x, wt, b))
    xs = torch.empty(n * h * w * c_store * 4, dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_f32_pack_input(xd.data_ptr(), xs.data_ptr(), n, c, h, w, c_store, None))
    packed = torch.empty(int(L.lib.ie_cuda_f32_packed_weight_bytes(d)), dtype=torch.uint8,
                         device="cuda")
    L.check(L.lib.ie_cuda_f32_pack_weights(d, wd.data_ptr(), packed.data_ptr(), None))
    m_store = (m + 15) // 16 * 16
    r_nhwc = np.zeros((n, h, w, m_store), np.float32)
    r_nhwc[..., :m] = r.transpose(0, 2, 3, 1)
    rd = torch.from_numpy(r_nhwc).cuda()
    y = torch.full((n, h, w, m_store), float("nan"), device="cuda")
    L.check(L.lib.ie_cuda_conv2d_bf16x3_residual(d, 1, xs.data_ptr(), packed.data_ptr(),
                                                 bd.data_ptr(), rd.data_ptr(), y.data_ptr(),
                                                 L.IE_Y_F32_NHWC, None))
    torch.cuda.synchronize()
    got = y.cpu().numpy()[..., :m]
    err = np.abs(got - want).max()
    assert err <= REL_TOL * np.abs(want).max(), err


def test_grouped_residual_rejected():
    import torch
    from computeengine_b200 import _lib as L
    from tests.qconv import desc_for
    d = desc_for(L, 1, 8, 5, 5, 8, 3, 3, pads=(1, 1, 1, 1), group=8, depthwise=1)
    t = torch.zeros(1024, device="cuda")
    rc = L.lib.ie_cuda_conv2d_f32_residual(d, 0, t.data_ptr(), t.data_ptr(), None, t.data_ptr(),
                                           t.data_ptr(), t.data_ptr(), 4096, None)
    assert rc == L.IE_UNSUPPORTED
