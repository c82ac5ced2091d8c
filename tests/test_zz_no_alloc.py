"""The no-allocation fp32 convolution entry point (ie_cuda_conv2d_f32_noalloc).

Some callers cannot allocate device memory or hand the library a workspace:
an operator whose forward() only receives the engine's host allocator, or a
host that forbids cudaMalloc / cudaFree because they synchronize the device
and disturb its own memory plan.  For them the library packs the operands
into a fixed scratch array in its own device image.  This test calls that
entry point through the C ABI twice in a row, on two different convolutions,
and compares each result with the regular entry point run on a caller-owned
workspace, within the fp32 path's tolerance (max |err| <= 1e-3 * max |ref|).
It also checks that a convolution too large for the scratch is rejected.

The file name sorts last so a run that stops at the first failure has
already run every other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def _desc(L, n, c, h, w, m, k, pad):
    from tests.qconv import desc_for
    return desc_for(L, n, c, h, w, m, k, k, (1, 1), (pad, pad, pad, pad))


def _run_pair(L, torch, n, c, h, w, m, k, pad, seed):
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)).cuda()
    wt = torch.from_numpy(rng.normal(0, 0.1, (m, c, k, k)).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.normal(0, 0.01, m).astype(np.float32)).cuda()
    d = _desc(L, n, c, h, w, m, k, pad)
    s = L.ConvShape()
    L.check(L.lib.ie_conv2d_resolve(d, m, s))
    stream = torch.cuda.current_stream().cuda_stream
    # regular entry point, workspace owned by the caller
    nbytes = int(L.lib.ie_cuda_conv2d_f32_workspace_bytes(d))
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    want = torch.full((n, m, s.out_h, s.out_w), float("nan"), device="cuda")
    L.check(L.lib.ie_cuda_conv2d_f32(d, L.IE_ACT_RELU, x.data_ptr(), wt.data_ptr(), b.data_ptr(),
                                     want.data_ptr(), ws.data_ptr(), nbytes, stream))
    # no-allocation entry point
    got = torch.full((n, m, s.out_h, s.out_w), float("nan"), device="cuda")
    L.check(L.lib.ie_cuda_conv2d_f32_noalloc(d, L.IE_ACT_RELU, x.data_ptr(), wt.data_ptr(),
                                             b.data_ptr(), got.data_ptr(), stream))
    torch.cuda.synchronize()
    return got.cpu().numpy(), want.cpu().numpy()


def test_noalloc_matches_regular_entry_point_twice():
    import torch
    from computeengine_b200 import _lib as L
    assert L.lib.ie_cuda_noalloc_scratch_bytes() == 16 << 20
    # two different convolutions back to back share the one scratch array
    for args in ((1, 64, 56, 56, 64, 3, 1, 0), (2, 24, 17, 19, 40, 5, 2, 1)):
        got, want = _run_pair(L, torch, *args)
        assert np.isfinite(got).all()
        err = float(np.abs(got - want).max())
        assert err <= REL_TOL * float(np.abs(want).max()), (args, err)
    assert L.take_device_error() == 0


def test_noalloc_matches_oracle_and_runs_grouped(oracle):
    """The regular entry point shares the pack and bf16x3 kernels with this
    one, so also check the no-allocation result against the fp32 oracle, and
    run a grouped convolution (CUDA-core path, which needs no scratch)."""
    import torch
    from computeengine_b200 import _lib as L
    from tests.qconv import desc_for
    rng = np.random.default_rng(17)
    stream = torch.cuda.current_stream().cuda_stream
    for (n, c, h, w, m, k, pad, group) in ((2, 32, 20, 18, 48, 3, 1, 1),
                                           (1, 32, 15, 15, 64, 3, 1, 4)):
        x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
        wt = rng.normal(0, 0.1, (m, c // group, k, k)).astype(np.float32)
        b = rng.normal(0, 0.01, m).astype(np.float32)
        d = desc_for(L, n, c, h, w, m, k, k, (1, 1), (pad,) * 4, (1, 1), group)
        s = L.ConvShape()
        L.check(L.lib.ie_conv2d_resolve(d, m, s))
        xd, wd, bd = (torch.from_numpy(a).cuda() for a in (x, wt, b))
        got = torch.full((n, m, s.out_h, s.out_w), float("nan"), device="cuda")
        L.check(L.lib.ie_cuda_conv2d_f32_noalloc(d, L.IE_ACT_NONE, xd.data_ptr(), wd.data_ptr(),
                                                 bd.data_ptr(), got.data_ptr(), stream))
        torch.cuda.synchronize()
        want = oracle.conv2d_f32(x, wt, b, pads=(pad,) * 4, group=group)
        err = float(np.abs(got.cpu().numpy() - want).max())
        assert err <= REL_TOL * float(np.abs(want).max()), (group, err)
    assert L.take_device_error() == 0


def test_noalloc_rejects_oversized_convolution():
    from computeengine_b200 import _lib as L
    d = _desc(L, 8, 64, 112, 112, 64, 3, 1)  # ~26 MB of packed activations
    need = int(L.lib.ie_cuda_conv2d_f32_workspace_bytes(d))
    assert need > int(L.lib.ie_cuda_noalloc_scratch_bytes())
    rc = L.lib.ie_cuda_conv2d_f32_noalloc(d, 0, None, None, None, None, None)
    assert rc == L.IE_INVALID_ARGUMENT
    assert b"scratch" in L.lib.ie_cuda_last_error()
