"""fp32 convolution on the B200 against the reference's own goldens and the
CPU oracle.  Dense convolutions run as bf16x3 on the tensor cores, grouped and
depthwise ones on CUDA cores.  Tolerance: max |err| <= 1e-3 * max |ref| for
bf16x3; 1e-5 absolute on the reference goldens (the reference test's own
tolerance, traditional_ops_test.cpp:99)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def run_f32(x, w, b=None, act=0, stride=(1, 1), pads=(0, 0, 0, 0), dil=(1, 1), group=1,
            auto_pad=0, depthwise=0):
    import torch
    from computeengine_b200 import _lib as L
    from tests.qconv import desc_for
    n, c, h, ww = x.shape
    m, _, kh, kw = w.shape
    d = desc_for(L, n, c, h, ww, m, kh, kw, stride, pads, dil, group, auto_pad, depthwise)
    s = L.ConvShape()
    L.check(L.lib.ie_conv2d_resolve(d, -1 if b is None else m, s))
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    wd = torch.from_numpy(np.ascontiguousarray(w, np.float32)).cuda()
    bd = torch.from_numpy(np.ascontiguousarray(b, np.float32)).cuda() if b is not None else None
    y = torch.full((n, m, s.out_h, s.out_w), float("nan"), device="cuda")
    nbytes = int(L.lib.ie_cuda_conv2d_f32_workspace_bytes(d))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_conv2d_f32(d, act, xd.data_ptr(), wd.data_ptr(),
                                     bd.data_ptr() if bd is not None else None, y.data_ptr(),
                                     ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert L.take_device_error() == 0
    return y.cpu().numpy()


def test_golden_conv(golden):
    # Dense convolutions run as bf16x3, whose split error is ~2^-16 relative
    # per product: the reference's 1e-5 absolute bound is at its edge, so the
    # fp32-path bound max|err| <= 1e-3 * max|ref| applies.
    want = golden["kConvExpected"]
    y = run_f32(golden["kConvInput"], golden["kConvWeight"], golden["kConvBias"], pads=(1, 1, 1, 1))
    assert np.abs(y - want).max() <= REL_TOL * np.abs(want).max()
    assert np.abs(y - want).max() <= 5e-5


def test_golden_depthwise(golden):
    y = run_f32(golden["kDepthwiseInput"], golden["kDepthwiseWeight"], golden["kDepthwiseBias"],
                group=2, depthwise=1)
    np.testing.assert_allclose(y, golden["kDepthwiseExpected"], atol=1e-5, rtol=0)


CASES = [
    # (n, c, h, w, m, kh, kw, stride, pads, group)
    (1, 64, 56, 56, 64, 3, 3, (1, 1), (1, 1, 1, 1), 1),     # single fp32 conv workload
    (2, 3, 32, 32, 64, 7, 7, (2, 2), (3, 3, 3, 3), 1),      # stem-like, c = 3
    (1, 256, 14, 14, 512, 1, 1, (2, 2), (0, 0, 0, 0), 1),   # strided projection
    (1, 32, 17, 19, 48, 3, 3, (1, 1), (0, 1, 2, 1), 1),     # asymmetric pads
    (1, 24, 10, 10, 48, 3, 3, (1, 1), (1, 1, 1, 1), 4),     # grouped (CUDA cores)
    (2, 32, 12, 12, 32, 3, 3, (2, 2), (1, 1, 1, 1), 32),    # depthwise stride 2
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(map(str, c[:7])) + f"_g{c[9]}")
def test_f32_matches_oracle(oracle, case):
    n, c, h, w, m, kh, kw, stride, pads, group = case
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / (c // group * kh * kw)), (m, c // group, kh, kw)).astype(np.float32)
    b = rng.normal(0, 0.01, m).astype(np.float32)
    got = run_f32(x, wt, b, act=1, stride=stride, pads=pads, group=group)
    want = oracle.conv2d_f32(x, wt, b, act=1, strides=stride, pads=pads, group=group, nthreads=8)
    err = np.abs(got - want).max()
    assert err <= REL_TOL * np.abs(want).max(), err


def test_config1_against_reference_conv(refconv):
    """The reference's own Conv2DOp on the single fp32 conv workload (seed 0)."""
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, (1, 64, 56, 56)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / 576), (64, 64, 3, 3)).astype(np.float32)
    b = rng.normal(0, 0.01, 64).astype(np.float32)
    rc, want = refconv.conv2d(x, wt, b, pads=(1, 1, 1, 1))
    assert rc == 0
    got = run_f32(x, wt, b, pads=(1, 1, 1, 1))
    err = np.abs(got - want).max()
    assert err <= REL_TOL * np.abs(want).max(), err


def test_f32_tile_policy_same_results(oracle):
    """An fp32 layer whose default tiles leave most SMs idle (deep K, small
    batch) takes narrower 128-position tiles under the fill policy; the
    products and their K order are the same, so both policies give the same
    floats, within tolerance of the oracle."""
    from computeengine_b200 import _lib as L
    from tests.qconv import tile_policy
    rng = np.random.default_rng(5)
    n, c, h, w, m = 2, 256, 14, 14, 256
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / (c * 9)), (m, c, 3, 3)).astype(np.float32)
    b = rng.normal(0, 0.01, m).astype(np.float32)
    with tile_policy(L.IE_TILE_DEFAULT):
        ref = run_f32(x, wt, b, act=1, pads=(1, 1, 1, 1))
        plan_d = L.last_plan()
    with tile_policy(L.IE_TILE_FILL):
        got = run_f32(x, wt, b, act=1, pads=(1, 1, 1, 1))
        plan_f = L.last_plan()
    assert plan_d.bn == 256 and plan_d.grid < 148
    assert plan_f.bn < plan_d.bn and plan_f.grid > plan_d.grid
    np.testing.assert_array_equal(got, ref)
    want = oracle.conv2d_f32(x, wt, b, act=1, pads=(1, 1, 1, 1), nthreads=8)
    assert np.abs(got - want).max() <= REL_TOL * np.abs(want).max()
