"""Single-layer convolution benchmark (the conv benchmark the reference's
src/benchmarks lacks: ie_bench.cpp only times the CPU matmul row kernel).

    python -m computeengine_b200.conv_bench --layer s1b1_conv3 [--batch 256] [--iters 50]
    python -m computeengine_b200.conv_bench --shape 256,64,56,56,256,1,1 --stride 1 --pad 0
    python -m computeengine_b200.conv_bench --layer s2b2_conv2 --dtype f32
    python -m computeengine_b200.conv_bench --layer stem   # the 4x1 layer of the stem re-layout

Times one layer of the ResNet-50 stack (or an explicit shape) with CUDA
events, after warm-up, and prints one JSON line: microseconds per launch,
TOPS (2 ops per MAC), algorithmic GB/s (input + output + weights once) and
the fractions of the measured peaks.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import numpy as np
import torch

from . import _lib as L
from .resnet import ConvLayer, resnet50_layers

ROOT = Path(__file__).resolve().parent.parent


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    d = json.loads(p.read_text()) if p.exists() else {}
    return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0)


def bench_layer(l: ConvLayer, batch: int, iters: int, dtype: str = "int8", seed: int = 0):
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(seed)
    d = L.ConvDesc()
    d.n, d.c, d.h, d.w, d.m, d.kh, d.kw = batch, l.cin, l.h, l.h, l.cout, l.k, l.k
    d.stride_h = d.stride_w = l.stride
    d.dil_h = d.dil_w = 1
    d.pad_top = d.pad_left = d.pad_bottom = d.pad_right = l.pad
    d.group = 1
    c_store = (l.cin + 15) // 16 * 16
    m_store = (l.cout + 15) // 16 * 16
    oh = l.out_h
    in_h, w_shape = l.h, (l.cout, l.cin, l.k, l.k)
    if l.name == "stem":
        # the 7x7 / 2 stem as the 4x1 layer over its space-to-depth re-layout
        # (the re-layout kernel itself is not timed here)
        if dtype != "int8":
            raise SystemExit("the stem re-layout is int8 only")
        L.check(L.lib.ie_cuda_q8_stem_desc(batch, l.cin, l.h, l.h, l.cout, d))
        in_h, c_store, w_shape = d.h, d.c, (l.cout, d.c, d.kh, d.kw)
    if dtype == "int8":
        x = torch.randint(0, 256, (batch, in_h, in_h, c_store), dtype=torch.uint8, device=dev)
        w = torch.from_numpy(rng.integers(-127, 128, w_shape).astype(np.int8)).to(dev)
        packed = torch.zeros(int(L.lib.ie_cuda_q8_packed_weight_bytes(d)), dtype=torch.uint8, device=dev)
        L.check(L.lib.ie_cuda_q8_pack_weights(d, w.data_ptr(), packed.data_ptr(), stream))
        bias = torch.zeros(l.cout, dtype=torch.int32, device=dev)
        mult = torch.full((l.cout,), 0.002, dtype=torch.float32, device=dev)
        y = torch.empty((batch, oh, oh, m_store), dtype=torch.uint8, device=dev)
        q = L.Q8Params()
        q.x_signed, q.zp_x, q.y_signed, q.zp_y, q.qmin, q.qmax = 0, 0, 0, 0, 0, 255

        def launch():
            L.check(L.lib.ie_cuda_conv2d_q8(d, q, x.data_ptr(), packed.data_ptr(), bias.data_ptr(),
                                            mult.data_ptr(), y.data_ptr(), stream))
        bytes_io = x.numel() + y.numel() + packed.numel()
    else:
        x = torch.randn((batch, l.h, l.h, 2 * c_store), device=dev).to(torch.bfloat16)
        w = torch.randn((l.cout, l.cin, l.k, l.k), device=dev)
        packed = torch.zeros(int(L.lib.ie_cuda_f32_packed_weight_bytes(d)), dtype=torch.uint8, device=dev)
        L.check(L.lib.ie_cuda_f32_pack_weights(d, w.data_ptr(), packed.data_ptr(), stream))
        bias = torch.zeros(l.cout, dtype=torch.float32, device=dev)
        y = torch.empty((batch, oh, oh, 2 * m_store), dtype=torch.bfloat16, device=dev)

        def launch():
            L.check(L.lib.ie_cuda_conv2d_bf16x3(d, L.IE_ACT_RELU, x.data_ptr(), packed.data_ptr(),
                                                bias.data_ptr(), y.data_ptr(), L.IE_Y_BF16X2_NHWC,
                                                stream))
        bytes_io = 2 * x.numel() + 2 * y.numel() + packed.numel()
    for _ in range(5):
        launch()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        launch()
    b.record()
    torch.cuda.synchronize()
    assert L.take_device_error() == 0
    us = a.elapsed_time(b) * 1e3 / iters
    macs = l.macs_per_image * batch
    hbm, bf16 = _peaks()
    tops = 2 * macs / us / 1e6
    peak = 2 * bf16 if dtype == "int8" else bf16 / 3
    return {"layer": l.name, "dtype": dtype, "batch": batch, "cin": l.cin, "cout": l.cout,
            "k": l.k, "stride": l.stride, "out": oh, "us": us, "tops": tops,
            "frac_tensor": tops / peak, "gbs": bytes_io / us / 1e3, "frac_hbm": bytes_io / us / 1e3 / hbm,
            "bound_us": max(2 * macs / (peak * 1e12) * 1e6, bytes_io / (hbm * 1e9) * 1e6)}


def _time(fn, iters: int) -> float:
    """Microseconds per call, CUDA events on the current stream after warm-up."""
    for _ in range(5):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    assert L.take_device_error() == 0
    return a.elapsed_time(b) * 1e3 / iters


def bench_configs(iters: int = 200) -> list:
    """The single-convolution workloads, each as its drop-in call on device
    tensors in the reference layout (NCHW), plus the int8 kernel alone:
      config 1: fp32 x U(-1,1) [1,64,56,56], w N(0, sqrt(2/576)) [64,64,3,3],
                bias N(0, 0.01), stride 1, pad 1, ReLU (ie_cuda_conv2d_f32);
      config 2: int8 x uint8 N(128,30) zp 128 [8,128,28,28], w U{-127..127}
                [128,128,3,3], per-channel multipliers, ReLU (pack input +
                ie_cuda_conv2d_q8 + unpack output, and the kernel alone)."""
    hbm, bf16 = _peaks()
    stream = torch.cuda.current_stream().cuda_stream
    dev = torch.device("cuda")
    out = []
    rng = np.random.default_rng(0)
    # config 1
    d = L.ConvDesc()
    d.n, d.c, d.h, d.w, d.m, d.kh, d.kw = 1, 64, 56, 56, 64, 3, 3
    d.stride_h = d.stride_w = d.dil_h = d.dil_w = 1
    d.pad_top = d.pad_left = d.pad_bottom = d.pad_right = 1
    d.group = 1
    x = torch.from_numpy(rng.uniform(-1, 1, (1, 64, 56, 56)).astype(np.float32)).to(dev)
    w = torch.from_numpy(rng.normal(0, np.sqrt(2 / 576), (64, 64, 3, 3)).astype(np.float32)).to(dev)
    b = torch.from_numpy(rng.normal(0, 0.01, 64).astype(np.float32)).to(dev)
    y = torch.empty((1, 64, 56, 56), device=dev)
    ws = torch.empty(int(L.lib.ie_cuda_conv2d_f32_workspace_bytes(d)), dtype=torch.uint8, device=dev)
    us = _time(lambda: L.check(L.lib.ie_cuda_conv2d_f32(d, L.IE_ACT_RELU, x.data_ptr(), w.data_ptr(),
                                                        b.data_ptr(), y.data_ptr(), ws.data_ptr(),
                                                        ws.numel(), stream)), iters)
    flops = 2 * 64 * 64 * 9 * 56 * 56
    # end to end through the operator API with host buffers: pinned H2D of x
    # and w, Conv2DOp.forward, pinned D2H of y, every call
    from .ops import Conv2DOp, QLinearConv2DOp
    op = Conv2DOp()
    op.configure({"pads": [1, 1, 1, 1], "activation": "RELU"})
    xh, wh, bh = (t.cpu().pin_memory() for t in (x, w, b))
    yh = torch.empty((1, 64, 56, 56)).pin_memory()
    xo, wo, bo = torch.empty_like(x), torch.empty_like(w), torch.empty_like(b)

    def op_e2e():
        xo.copy_(xh, non_blocking=True)
        wo.copy_(wh, non_blocking=True)
        bo.copy_(bh, non_blocking=True)
        res = [None]
        assert op.forward([xo, wo, bo], res)
        yh.copy_(res[0], non_blocking=True)
    us_e2e = _time(op_e2e, iters)
    out.append({"config": 1, "workload": "fp32 conv [1,64,56,56] 3x3 -> 64, ReLU, NCHW drop-in "
                "(pack input + pack weights + bf16x3 conv)", "us": us,
                "gflops": flops / us / 1e3, "frac_of_bf16_peak_over_3": flops / us / 1e6 / (bf16 / 3),
                "e2e_us": us_e2e, "e2e": "Conv2DOp.forward with host buffers (pinned H2D of x, w, b "
                                         "and D2H of y inside the timed region)"})
    # config 2
    d2 = L.ConvDesc()
    d2.n, d2.c, d2.h, d2.w, d2.m, d2.kh, d2.kw = 8, 128, 28, 28, 128, 3, 3
    d2.stride_h = d2.stride_w = d2.dil_h = d2.dil_w = 1
    d2.pad_top = d2.pad_left = d2.pad_bottom = d2.pad_right = 1
    d2.group = 1
    xq = torch.from_numpy(np.clip(np.rint(rng.normal(128, 30, (8, 128, 28, 28))), 0, 255)
                          .astype(np.uint8)).to(dev)
    wq = torch.from_numpy(rng.integers(-127, 128, (128, 128, 3, 3)).astype(np.int8)).to(dev)
    packed = torch.zeros(int(L.lib.ie_cuda_q8_packed_weight_bytes(d2)), dtype=torch.uint8, device=dev)
    L.check(L.lib.ie_cuda_q8_pack_weights(d2, wq.data_ptr(), packed.data_ptr(), stream))
    bq = torch.from_numpy(np.rint(rng.normal(0, 500, 128)).astype(np.int32)).to(dev)
    mult = torch.from_numpy((0.02 * rng.uniform(0.001, 0.01, 128) / 0.05).astype(np.float32)).to(dev)
    x_nhwc = torch.empty((8, 28, 28, 128), dtype=torch.uint8, device=dev)
    y_nhwc = torch.empty((8, 28, 28, 128), dtype=torch.uint8, device=dev)
    y_nchw = torch.empty((8, 128, 28, 28), dtype=torch.uint8, device=dev)
    q = L.Q8Params()
    q.x_signed, q.zp_x, q.y_signed, q.zp_y, q.qmin, q.qmax = 1, 0, 0, 0, 0, 255

    def conv_only():
        L.check(L.lib.ie_cuda_conv2d_q8(d2, q, x_nhwc.data_ptr(), packed.data_ptr(), bq.data_ptr(),
                                        mult.data_ptr(), y_nhwc.data_ptr(), stream))

    def drop_in():
        L.check(L.lib.ie_cuda_q8_pack_input(xq.data_ptr(), x_nhwc.data_ptr(), 8, 128, 28, 28, 128,
                                            0x80, stream))
        conv_only()
        L.check(L.lib.ie_cuda_q8_unpack_output(y_nhwc.data_ptr(), y_nchw.data_ptr(), 8, 128, 28, 28,
                                               128, stream))
    ops = 2 * 8 * 128 * 128 * 9 * 28 * 28
    us_k = _time(conv_only, iters)
    us_d = _time(drop_in, iters)
    qop = QLinearConv2DOp()
    qop.configure({"pads": [1, 1, 1, 1], "multiplier": [float(v) for v in mult.cpu().numpy()],
                   "x_zero_point": 128, "y_zero_point": 0, "qmin": 0, "qmax": 255})
    xqh, wqh, bqh = (t.cpu().pin_memory() for t in (xq, wq, bq))
    yqh = torch.empty((8, 128, 28, 28), dtype=torch.uint8).pin_memory()
    xqo, wqo, bqo = torch.empty_like(xq), torch.empty_like(wq), torch.empty_like(bq)

    def qop_e2e():
        xqo.copy_(xqh, non_blocking=True)
        wqo.copy_(wqh, non_blocking=True)
        bqo.copy_(bqh, non_blocking=True)
        res = [None]
        assert qop.forward([xqo, wqo, bqo], res)
        yqh.copy_(res[0], non_blocking=True)
    us_qe = _time(qop_e2e, iters)
    out.append({"config": 2, "workload": "int8 conv [8,128,28,28] 3x3 -> 128, requantized, ReLU",
                "kernel_us": us_k, "kernel_tops": ops / us_k / 1e6,
                "frac_of_2x_bf16_peak": ops / us_k / 1e6 / (2 * bf16),
                "drop_in_us": us_d, "drop_in_tops": ops / us_d / 1e6,
                "e2e_us": us_qe, "e2e": "QLinearConv2DOp.forward with host buffers (pinned H2D of "
                                        "x, w, bias and D2H of y inside the timed region)"})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layer", action="append", default=[])
    ap.add_argument("--all", action="store_true")
    ap.add_argument("--shape", help="n,c,h,w,m,kh,kw")
    ap.add_argument("--stride", type=int, default=1)
    ap.add_argument("--pad", type=int, default=0)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--dtype", choices=["int8", "f32"], default="int8")
    ap.add_argument("--configs", action="store_true",
                    help="time the single-convolution workloads (configs 1 and 2)")
    a = ap.parse_args()
    if a.configs:
        for r in bench_configs():
            print(json.dumps(r), flush=True)
        return
    layers = {l.name: l for l in resnet50_layers()}
    todo = []
    if a.shape:
        n, c, h, w, m, kh, kw = (int(v) for v in a.shape.split(","))
        todo.append((ConvLayer("custom", c, m, kh, a.stride, a.pad, h, "x"), n))
    names = list(layers) if a.all else a.layer
    for name in names:
        if name == "stem" and a.dtype != "int8":
            continue  # the stem re-layout is int8 only
        todo.append((layers[name], a.batch))
    for l, n in todo:
        print(json.dumps(bench_layer(l, n, a.iters, a.dtype)), flush=True)


if __name__ == "__main__":
    main()
