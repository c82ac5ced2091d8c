"""MobileNetV2-style int8 inverted-residual block sweep on the B200 kernels.

The standard 17-block schedule (t, c, n, s) = (1,16,1,1), (6,24,2,2),
(6,32,3,2), (6,64,4,2), (6,96,3,1), (6,160,3,2), (6,320,1,1) over a
[N, 32, 112, 112] uint8 input (zero point 128, scale 0.02).  Each block is
1x1 expand (skipped when t == 1) -> 3x3 depthwise (stride s on the first block
of a group) -> 1x1 project.  The reference runs such graphs through Conv2DOp
and DepthwiseConv2DOp (src/ops/traditional/conv2d_op.h:36-67); here the 1x1
convolutions run on the tensor-core implicit GEMM and the depthwise ones on
the bandwidth-bound NHWC kernel.  Residual additions are not part of the
sweep.

Quantization: per-channel int8 weights U{-127..127} with scales
U(0.001, 0.01), int32 bias N(0, 500).  Expand and depthwise outputs are uint8
with scale 0.05, zero point 0 and ReLU6 folded in (qmax = round(6 / 0.05) =
120); project outputs are linear int8 (scale 0.05, zero point 0), which the
next block's expand reads directly.
"""
from __future__ import annotations

import argparse
import json
from dataclasses import dataclass
from typing import Dict, List, Optional

import numpy as np

IN_SCALE, IN_ZP = 0.02, 128
ACT_SCALE = 0.05
RELU6_QMAX = 120
SCHEDULE = ((1, 16, 1, 1), (6, 24, 2, 2), (6, 32, 3, 2), (6, 64, 4, 2), (6, 96, 3, 1),
            (6, 160, 3, 2), (6, 320, 1, 1))


@dataclass
class Layer:
    name: str
    kind: str        # "expand" | "dw" | "project"
    cin: int
    cout: int
    k: int
    stride: int
    h: int           # input height (= width)
    src: str
    s_x: float
    zp_x: int
    x_signed: bool
    y_signed: bool
    qmax: int

    @property
    def out_h(self) -> int:
        pad = self.k // 2
        return (self.h + 2 * pad - self.k) // self.stride + 1

    @property
    def macs_per_image(self) -> int:
        per_out = self.k * self.k * (1 if self.kind == "dw" else self.cin)
        return self.out_h * self.out_h * self.cout * per_out


def mobilenetv2_layers(image: int = 112, cin: int = 32) -> List[Layer]:
    layers: List[Layer] = []
    h, src, s_x, zp_x, signed = image, "input", IN_SCALE, IN_ZP, False
    b = 0
    for t, c, n, s in SCHEDULE:
        for i in range(n):
            stride = s if i == 0 else 1
            p = f"b{b:02d}"
            hidden = cin * t
            if t != 1:
                layers.append(Layer(p + "_expand", "expand", cin, hidden, 1, 1, h, src, s_x, zp_x,
                                    signed, False, RELU6_QMAX))
                src, s_x, zp_x, signed = p + "_expand", ACT_SCALE, 0, False
            dw = Layer(p + "_dw", "dw", hidden, hidden, 3, stride, h, src, s_x, zp_x, signed, False,
                       RELU6_QMAX)
            layers.append(dw)
            h = dw.out_h
            layers.append(Layer(p + "_project", "project", hidden, c, 1, 1, h, dw.name, ACT_SCALE, 0,
                                False, True, 127))
            src, s_x, zp_x, signed, cin = p + "_project", ACT_SCALE, 0, True, c
            b += 1
    assert b == 17
    return layers


@dataclass
class QParams:
    w: np.ndarray
    bias: np.ndarray
    mult: np.ndarray


def make_params(layers: List[Layer], seed: int = 0) -> Dict[str, QParams]:
    out = {}
    for i, l in enumerate(layers):
        rng = np.random.default_rng([seed, 7, i])
        cw = 1 if l.kind == "dw" else l.cin
        w = rng.integers(-127, 128, (l.cout, cw, l.k, l.k), dtype=np.int64).astype(np.int8)
        s_w = rng.uniform(0.001, 0.01, l.cout).astype(np.float32)
        bias = np.rint(rng.normal(0.0, 500.0, l.cout)).astype(np.int32)
        mult = ((np.float64(l.s_x) * s_w.astype(np.float64)) / np.float64(ACT_SCALE)).astype(np.float32)
        out[l.name] = QParams(w, bias, mult)
    return out


def make_input(batch: int, seed: int = 0, image: int = 112, c: int = 32) -> np.ndarray:
    rng = np.random.default_rng([seed, 11])
    return np.clip(np.rint(rng.normal(128.0, 30.0, (batch, c, image, image))), 0, 255).astype(np.uint8)


def _c16(c: int) -> int:
    return (c + 15) // 16 * 16


class MobileNetV2Q8:
    """The sweep resident on one GPU; run(x) leaves every layer's NHWC output
    (channels padded to 16) in ``acts``."""

    def __init__(self, batch: int, params: Dict[str, QParams], device="cuda", image: int = 112):
        import torch

        from . import _lib as L
        self.L, self.torch = L, torch
        self.batch, self.image = batch, image
        self.device = torch.device(device)
        self.layers = mobilenetv2_layers(image)
        dev = self.device
        stream = torch.cuda.current_stream(dev).cuda_stream
        self.descs, self.packed, self.bias, self.mult, self.qp, self.acts = {}, {}, {}, {}, {}, {}
        for l in self.layers:
            p = params[l.name]
            d = L.ConvDesc()
            d.n, d.c, d.h, d.w, d.m, d.kh, d.kw = batch, l.cin, l.h, l.h, l.cout, l.k, l.k
            d.stride_h = d.stride_w = l.stride
            d.dil_h = d.dil_w = 1
            d.pad_top = d.pad_left = d.pad_bottom = d.pad_right = l.k // 2
            w_dev = torch.from_numpy(p.w).to(dev)
            if l.kind == "dw":
                d.group, d.depthwise = l.cin, 1
                nbytes = int(L.lib.ie_cuda_dw_q8_packed_weight_bytes(d))
                packed = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
                L.check(L.lib.ie_cuda_dw_q8_pack_weights(d, w_dev.data_ptr(), packed.data_ptr(), stream))
            else:
                d.group = 1
                nbytes = int(L.lib.ie_cuda_q8_packed_weight_bytes(d))
                packed = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
                L.check(L.lib.ie_cuda_q8_pack_weights(d, w_dev.data_ptr(), packed.data_ptr(), stream))
            q = L.Q8Params()
            q.x_signed, q.zp_x = int(l.x_signed), l.zp_x
            q.y_signed, q.zp_y = int(l.y_signed), 0
            q.qmin, q.qmax = (-128, 127) if l.y_signed else (0, l.qmax)
            self.descs[l.name], self.packed[l.name], self.qp[l.name] = d, packed, q
            self.bias[l.name] = torch.from_numpy(p.bias).to(dev)
            self.mult[l.name] = torch.from_numpy(p.mult).to(dev)
            self.acts[l.name] = torch.empty((batch, l.out_h, l.out_h, _c16(l.cout)), dtype=torch.uint8,
                                            device=dev)
        self.x_nhwc = torch.empty((batch, image, image, 32), dtype=torch.uint8, device=dev)
        self.graph = None
        torch.cuda.synchronize(dev)

    def run(self, x_u8_nchw) -> int:
        L = self.L
        stream = self.torch.cuda.current_stream(self.device).cuda_stream
        L.check(L.lib.ie_cuda_q8_pack_input(x_u8_nchw.data_ptr(), self.x_nhwc.data_ptr(), self.batch,
                                            32, self.image, self.image, 32, 0, stream))
        n = 1
        for l in self.layers:
            src = self.x_nhwc if l.src == "input" else self.acts[l.src]
            fn = L.lib.ie_cuda_dwconv2d_q8 if l.kind == "dw" else L.lib.ie_cuda_conv2d_q8
            L.check(fn(self.descs[l.name], self.qp[l.name], src.data_ptr(),
                       self.packed[l.name].data_ptr(), self.bias[l.name].data_ptr(),
                       self.mult[l.name].data_ptr(), self.acts[l.name].data_ptr(), stream))
            n += 1
        return n

    def capture(self, x):
        torch = self.torch
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.launches = self.run(x)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.run(x)
        torch.cuda.synchronize(self.device)


def hbm_bytes_per_image(layers: List[Layer]) -> Dict[str, int]:
    """Algorithmic bytes per image: each layer reads its input and writes its
    output once (uint8 / int8), weights excluded (shared by the batch)."""
    tot = {"all": 0, "dw": 0}
    for l in layers:
        b = l.h * l.h * l.cin + l.out_h * l.out_h * l.cout
        tot["all"] += b
        if l.kind == "dw":
            tot["dw"] += b
    return tot


def benchmark(batch: int = 64, iters: int = 50) -> dict:
    """Times the sweep (CUDA-graph replays) and each depthwise layer."""
    import torch
    layers = mobilenetv2_layers()
    params = make_params(layers)
    net = MobileNetV2Q8(batch, params)
    x = torch.from_numpy(make_input(batch)).cuda()
    net.capture(x)
    for _ in range(5):
        net.graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        net.graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    macs = sum(l.macs_per_image for l in layers) * batch
    by = hbm_bytes_per_image(layers)
    return {"workload": "MobileNetV2 int8 inverted-residual sweep (17 blocks)", "batch": batch,
            "ms_per_step": ms, "tops": 2 * macs / ms / 1e9, "images_per_s": batch / ms * 1e3,
            "algorithmic_gbs": by["all"] * batch / ms / 1e6, "launches": net.launches}


def layer_times(batch: int = 64, iters: int = 20, only: Optional[str] = None) -> List[dict]:
    """Times every launch of the sweep on its own (CUDA events around each
    launch, averaged over `iters` passes); bytes are the algorithmic bytes of
    that layer (input + output once).  `only` restricts it to one layer (its
    input is still produced by running the sweep once)."""
    import torch
    layers = mobilenetv2_layers()
    net = MobileNetV2Q8(batch, make_params(layers))
    x = torch.from_numpy(make_input(batch)).cuda()
    L = net.L
    stream = torch.cuda.current_stream().cuda_stream
    net.run(x)
    torch.cuda.synchronize()
    out = []
    for l in layers:
        if only is not None and l.name != only:
            continue
        src = net.x_nhwc if l.src == "input" else net.acts[l.src]
        fn = L.lib.ie_cuda_dwconv2d_q8 if l.kind == "dw" else L.lib.ie_cuda_conv2d_q8
        args = (net.descs[l.name], net.qp[l.name], src.data_ptr(), net.packed[l.name].data_ptr(),
                net.bias[l.name].data_ptr(), net.mult[l.name].data_ptr(),
                net.acts[l.name].data_ptr(), stream)
        for _ in range(3):
            L.check(fn(*args))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            L.check(fn(*args))
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / iters
        by = batch * (l.h * l.h * _c16(l.cin) + l.out_h * l.out_h * _c16(l.cout))
        out.append({"layer": l.name, "kind": l.kind, "cin": l.cin, "cout": l.cout, "h": l.h,
                    "stride": l.stride, "us": us, "gbs": by / us / 1e3})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--layers", action="store_true", help="also time each launch on its own")
    ap.add_argument("--only", help="time this one layer (e.g. b02_dw) and nothing else")
    a = ap.parse_args()
    if a.only:
        for r in layer_times(a.batch, a.iters, a.only):
            print(json.dumps(r))
        return
    print(json.dumps(benchmark(a.batch, a.iters)))
    if a.layers:
        for r in layer_times(a.batch):
            print(json.dumps(r))


if __name__ == "__main__":
    main()
