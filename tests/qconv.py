"""Helpers shared by the int8 tests: seeded quantized problems and runners
that call the CUDA kernels through the C ABI (ctypes) with torch-owned device
buffers."""
from __future__ import annotations

from contextlib import contextmanager

import numpy as np


def make_q8_problem(rng, n, c, h, w, m, kh, kw, *, x_zp=128, x_signed=False, x_std=30.0,
                    s_x=0.02, s_y=0.05, zp_y=0, bias_std=500.0, with_bias=True, group=1):
    """Seeded int8 conv problem in the benchmark's int8 scheme: uint8 activations with a zero
    point, per-channel int8 weights, int32 bias, fp32 multipliers (NCHW host arrays)."""
    if x_signed:
        x = np.clip(np.rint(rng.normal(0, x_std, (n, c, h, w))), -128, 127).astype(np.int8)
    else:
        x = np.clip(np.rint(rng.normal(x_zp, x_std, (n, c, h, w))), 0, 255).astype(np.uint8)
    wq = rng.integers(-127, 128, (m, c // group, kh, kw), dtype=np.int64).astype(np.int8)
    s_w = rng.uniform(0.001, 0.01, m).astype(np.float32)
    mult = ((np.float64(s_x) * s_w.astype(np.float64)) / np.float64(s_y)).astype(np.float32)
    bias = np.rint(rng.normal(0, bias_std, m)).astype(np.int32) if with_bias else None
    return x, wq, bias, mult


def desc_for(L, n, c, h, w, m, kh, kw, stride=(1, 1), pads=(0, 0, 0, 0), dil=(1, 1), group=1,
             auto_pad=0, depthwise=0):
    d = L.ConvDesc()
    d.n, d.c, d.h, d.w, d.m, d.kh, d.kw = n, c, h, w, m, kh, kw
    d.stride_h, d.stride_w = stride
    d.dil_h, d.dil_w = dil
    d.pad_top, d.pad_left, d.pad_bottom, d.pad_right = pads
    d.group = group
    d.auto_pad = auto_pad
    d.depthwise = depthwise
    return d


def run_conv_q8_gpu(x, wq, bias, mult, *, stride=(1, 1), pads=(0, 0, 0, 0), dil=(1, 1),
                    zp_x=128, zp_y=0, qmin=0, qmax=255, raw_acc=False, device="cuda",
                    y_signed=False, force_halo=False):
    """Runs ie_cuda_conv2d_q8 (or _acc) on NCHW host arrays, returns NCHW host output.

    uint8 with zero point 128 goes through the XOR re-basing (int8, zero point
    0); any other nonzero zero point (or force_halo) through the haloed input
    whose padding holds the zero point."""
    import torch
    from computeengine_b200 import _lib as L

    n, c, h, w = x.shape
    m, _, kh, kw = wq.shape
    d = desc_for(L, n, c, h, w, m, kh, kw, stride, pads, dil)
    s = L.ConvShape()
    L.check(L.lib.ie_conv2d_resolve(d, -1 if bias is None else m, s))
    c_store = (c + 15) // 16 * 16
    m_store = (m + 15) // 16 * 16
    stream = torch.cuda.current_stream().cuda_stream
    x_dev = torch.from_numpy(np.ascontiguousarray(x)).to(device)
    x_nhwc = torch.zeros((n, h, w, c_store), dtype=torch.uint8, device=device)
    q = L.Q8Params()
    q.y_signed, q.zp_y, q.qmin, q.qmax = int(y_signed), zp_y, qmin, qmax
    if x.dtype == np.uint8 and zp_x == 128 and not force_halo:
        xor, q.x_signed, q.zp_x = 0x80, 1, 0
    else:
        xor, q.x_signed, q.zp_x = 0, int(x.dtype == np.int8), zp_x
    if q.zp_x != 0:
        hb = int(L.lib.ie_cuda_q8_halo_input_bytes(d))
        assert hb > 0
        x_nhwc = torch.full((hb,), 0x5A, dtype=torch.uint8, device=device)
        L.check(L.lib.ie_cuda_q8_pack_input_halo(d, x_dev.data_ptr(), x_nhwc.data_ptr(), q.zp_x,
                                                 stream))
    else:
        L.check(L.lib.ie_cuda_q8_pack_input(x_dev.data_ptr(), x_nhwc.data_ptr(), n, c, h, w,
                                            c_store, xor, stream))
    w_dev = torch.from_numpy(np.ascontiguousarray(wq)).to(device)
    packed = torch.zeros(int(L.lib.ie_cuda_q8_packed_weight_bytes(d)), dtype=torch.uint8,
                         device=device)
    L.check(L.lib.ie_cuda_q8_pack_weights(d, w_dev.data_ptr(), packed.data_ptr(), stream))
    b_dev = torch.from_numpy(bias).to(device) if bias is not None else None
    m_dev = torch.from_numpy(mult).to(device)
    if raw_acc:
        y = torch.full((n, s.out_h, s.out_w, m_store), -7, dtype=torch.int32, device=device)
        L.check(L.lib.ie_cuda_conv2d_q8_acc(d, q, x_nhwc.data_ptr(), packed.data_ptr(),
                                            b_dev.data_ptr() if b_dev is not None else None,
                                            y.data_ptr(), stream))
    else:
        y = torch.full((n, s.out_h, s.out_w, m_store), 77, dtype=torch.uint8, device=device)
        L.check(L.lib.ie_cuda_conv2d_q8(d, q, x_nhwc.data_ptr(), packed.data_ptr(),
                                        b_dev.data_ptr() if b_dev is not None else None,
                                        m_dev.data_ptr(), y.data_ptr(), stream))
    torch.cuda.synchronize()
    assert L.take_device_error() == 0
    out = y[..., :m].permute(0, 3, 1, 2).contiguous().cpu().numpy()
    return out.view(np.int8) if (y_signed and not raw_acc) else out


@contextmanager
def tile_policy(policy: int):
    """Runs the block under an int8 tile policy (ie_cuda_set_tile_policy) and
    restores the previous one."""
    from computeengine_b200 import _lib as L
    prev = L.set_tile_policy(policy)
    try:
        yield
    finally:
        L.set_tile_policy(prev)
