"""Single-layer convolution benchmark (the conv benchmark the reference's
src/benchmarks lacks: ie_bench.cpp only times the CPU matmul row kernel).

    python -m computeengine_b200.conv_bench --layer s1b1_conv3 [--batch 256] [--iters 50]
    python -m computeengine_b200.conv_bench --shape 256,64,56,56,256,1,1 --stride 1 --pad 0
    python -m computeengine_b200.conv_bench --layer s2b2_conv2 --dtype f32

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
    if dtype == "int8":
        x = torch.randint(0, 256, (batch, l.h, l.h, c_store), dtype=torch.uint8, device=dev)
        w = torch.from_numpy(rng.integers(-127, 128, (l.cout, l.cin, l.k, l.k)).astype(np.int8)).to(dev)
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
    a = ap.parse_args()
    layers = {l.name: l for l in resnet50_layers()}
    todo = []
    if a.shape:
        n, c, h, w, m, kh, kw = (int(v) for v in a.shape.split(","))
        todo.append((ConvLayer("custom", c, m, kh, a.stride, a.pad, h, "x"), n))
    names = list(layers) if a.all else a.layer
    for name in names:
        if name == "stem":
            continue  # the stem runs through its own re-layout; see bench.py
        todo.append((layers[name], a.batch))
    for l, n in todo:
        print(json.dumps(bench_layer(l, n, a.iters, a.dtype)), flush=True)


if __name__ == "__main__":
    main()
