"""ResNet-50 v1.5 convolution stack on the B200 kernels (int8 and fp32).

The 53 convolutions of ResNet-50 v1.5: a 7x7/2 stem, bottleneck blocks
1x1 -> 3x3 -> 1x1 in stages [3, 4, 6, 3] with widths 64/128/256/512 (x4
expansion), the stride on the 3x3 of each stage's first block and a 1x1
projection (downsample) beside it.  The reference runs such a graph node by
node on the CPU (Executor::run, src/core/runtime/executor.cpp:53-83, with
Conv2DOp at conv2d_op.cpp:73); here every node is one launch of the
implicit-GEMM kernel, captured once into a CUDA graph.

Stack definition (what the benchmark counts): each main-path conv consumes the
previous conv's output, each projection consumes its block's input, and the
stage-1 input is the 3x3/2 max pool of the stem output.  Residual additions
are not part of the stack.

int8 scheme per layer: per-output-channel symmetric int8 weights
U{-127..127} with scales U(0.001, 0.01), int32 bias N(0, 500), uint8
activations (the network input has zero point 128 and scale 0.02; every conv
output has zero point 0 and scale 0.05 with ReLU folded), multiplier
s_x * s_w[m] / s_y computed in double and rounded to fp32.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

IN_SCALE, IN_ZP = 0.02, 128
ACT_SCALE = 0.05


@dataclass
class ConvLayer:
    name: str
    cin: int
    cout: int
    k: int
    stride: int
    pad: int
    h: int           # input height (= width)
    src: str         # name of the tensor this layer reads
    out_h: int = 0

    def __post_init__(self):
        self.out_h = (self.h + 2 * self.pad - self.k) // self.stride + 1

    @property
    def macs_per_image(self) -> int:
        return self.out_h * self.out_h * self.cout * self.cin * self.k * self.k


def resnet50_layers(image: int = 224) -> List[ConvLayer]:
    layers = [ConvLayer("stem", 3, 64, 7, 2, 3, image, "input")]
    h = layers[0].out_h // 2  # after the 3x3/2 max pool
    prev, cin = "pool", 64
    for si, (blocks, width) in enumerate(zip((3, 4, 6, 3), (64, 128, 256, 512))):
        cout = width * 4
        for bi in range(blocks):
            stride = 2 if (bi == 0 and si > 0) else 1
            p = f"s{si + 1}b{bi + 1}"
            block_in = prev
            layers.append(ConvLayer(p + "_conv1", cin, width, 1, 1, 0, h, block_in))
            layers.append(ConvLayer(p + "_conv2", width, width, 3, stride, 1, h, p + "_conv1"))
            h2 = layers[-1].out_h
            layers.append(ConvLayer(p + "_conv3", width, cout, 1, 1, 0, h2, p + "_conv2"))
            if bi == 0:
                layers.append(ConvLayer(p + "_down", cin, cout, 1, stride, 0, h, block_in))
            prev, cin, h = p + "_conv3", cout, h2
    assert len(layers) == 53
    return layers


def macs_per_image(layers: Optional[List[ConvLayer]] = None) -> int:
    return sum(l.macs_per_image for l in (layers or resnet50_layers()))


@dataclass
class QuantLayerParams:
    w: np.ndarray        # int8 [cout, cin, k, k]
    bias: np.ndarray     # int32 [cout]
    mult: np.ndarray     # fp32 [cout]
    s_w: np.ndarray      # fp32 [cout]
    s_x: float
    zp_x: int


def make_q8_params(layers: List[ConvLayer], seed: int = 0) -> Dict[str, QuantLayerParams]:
    """Seeded int8 weights, biases and requantize multipliers for every layer."""
    params = {}
    for i, l in enumerate(layers):
        rng = np.random.default_rng([seed, i])
        w = rng.integers(-127, 128, (l.cout, l.cin, l.k, l.k), dtype=np.int64).astype(np.int8)
        s_w = rng.uniform(0.001, 0.01, l.cout).astype(np.float32)
        bias = np.rint(rng.normal(0.0, 500.0, l.cout)).astype(np.int32)
        s_x = IN_SCALE if l.src == "input" else ACT_SCALE
        zp_x = IN_ZP if l.src == "input" else 0
        mult = ((np.float64(s_x) * s_w.astype(np.float64)) / np.float64(ACT_SCALE)).astype(np.float32)
        params[l.name] = QuantLayerParams(w, bias, mult, s_w, s_x, zp_x)
    return params


def make_input_u8(batch: int, seed: int = 0, image: int = 224) -> np.ndarray:
    """uint8 NCHW input, round(N(128, 30)) clamped to 0..255."""
    rng = np.random.default_rng([seed, 1 << 20])
    x = rng.normal(128.0, 30.0, (batch, 3, image, image))
    return np.clip(np.rint(x), 0, 255).astype(np.uint8)


class ResNet50Q8:
    """int8 ResNet-50 conv stack resident on one GPU.

    ``run(x)`` takes a uint8 NCHW device tensor [batch, 3, 224, 224] and leaves
    every layer's NHWC uint8 output in ``self.acts``.  All buffers are
    allocated once; ``capture()`` records the whole stack into a CUDA graph.
    """

    def __init__(self, batch: int, params: Dict[str, QuantLayerParams], device="cuda",
                 image: int = 224, weights_from_rank0: bool = False):
        import torch

        from . import _lib as L

        self.L = L
        self.torch = torch
        self.batch = batch
        self.device = torch.device(device)
        self.layers = resnet50_layers(image)
        self.image = image
        dev = self.device
        stream = torch.cuda.current_stream(dev).cuda_stream
        self.descs = {}
        self.packed = {}
        self.bias = {}
        self.mult = {}
        self.acts = {}
        self.qp = {}
        for l in self.layers:
            p = params[l.name]
            if l.name == "stem":
                d = L.ConvDesc()
                L.check(L.lib.ie_cuda_q8_stem_desc(batch, l.cin, image, image, l.cout, d))
                nbytes = int(L.lib.ie_cuda_q8_packed_weight_bytes(d))
                packed = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
                w_dev = torch.from_numpy(p.w).to(dev)
                L.check(L.lib.ie_cuda_q8_stem_pack_weights(w_dev.data_ptr(), packed.data_ptr(),
                                                           l.cout, l.cin, stream))
            else:
                d = L.ConvDesc()
                d.n, d.c, d.h, d.w, d.m, d.kh, d.kw = batch, l.cin, l.h, l.h, l.cout, l.k, l.k
                d.stride_h = d.stride_w = l.stride
                d.dil_h = d.dil_w = 1
                d.pad_top = d.pad_left = d.pad_bottom = d.pad_right = l.pad
                d.group = 1
                nbytes = int(L.lib.ie_cuda_q8_packed_weight_bytes(d))
                packed = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
                w_dev = torch.from_numpy(p.w).to(dev)
                L.check(L.lib.ie_cuda_q8_pack_weights(d, w_dev.data_ptr(), packed.data_ptr(),
                                                      stream))
            self.descs[l.name] = d
            self.packed[l.name] = packed
            self.bias[l.name] = torch.from_numpy(p.bias).to(dev)
            self.mult[l.name] = torch.from_numpy(p.mult).to(dev)
            q = L.Q8Params()
            q.x_signed = 1 if l.src == "input" else 0  # the stem input is re-based to int8
            q.zp_x, q.y_signed, q.zp_y, q.qmin, q.qmax = 0, 0, 0, 0, 255
            self.qp[l.name] = q
            self.acts[l.name] = torch.empty((batch, l.out_h, l.out_h, l.cout), dtype=torch.uint8,
                                            device=dev)
        stem = self.layers[0]
        self.stem_in = torch.empty((batch, image // 2, image // 2, 64), dtype=torch.uint8,
                                   device=dev)
        ph = (stem.out_h + 2 - 3) // 2 + 1
        self.acts["pool"] = torch.empty((batch, ph, ph, 64), dtype=torch.uint8, device=dev)
        self.graph = None
        self.static_input = None
        torch.cuda.synchronize(dev)

    @property
    def output(self):
        return self.acts[self.layers[-1].name]

    def tensors(self):
        """Every device tensor holding weights or parameters (for broadcast)."""
        out = []
        for l in self.layers:
            out += [self.packed[l.name], self.bias[l.name], self.mult[l.name]]
        return out

    def run(self, x_u8_nchw) -> int:
        """Launches the whole stack on the current stream; returns the number of
        kernel launches issued."""
        L = self.L
        stream = self.torch.cuda.current_stream(self.device).cuda_stream
        n = 0
        b, img = self.batch, self.image
        L.check(L.lib.ie_cuda_q8_stem_pack_input(x_u8_nchw.data_ptr(), self.stem_in.data_ptr(), b,
                                                 3, img, img, 0x80, stream))
        n += 1
        for l in self.layers:
            if l.src == "input":
                src = self.stem_in
            else:
                src = self.acts[l.src]
            L.check(L.lib.ie_cuda_conv2d_q8(self.descs[l.name], self.qp[l.name], src.data_ptr(),
                                            self.packed[l.name].data_ptr(),
                                            self.bias[l.name].data_ptr(),
                                            self.mult[l.name].data_ptr(),
                                            self.acts[l.name].data_ptr(), stream))
            n += 1
            if l.name == "stem":
                s = self.acts["stem"]
                L.check(L.lib.ie_cuda_q8_maxpool2d(s.data_ptr(), self.acts["pool"].data_ptr(), b,
                                                   s.shape[1], s.shape[2], 64, 3, 2, 1, 0, stream))
                n += 1
        return n

    def capture(self, x_u8_nchw):
        """Records run(x) into a CUDA graph; replay() re-runs it on the same
        input buffer."""
        torch = self.torch
        self.static_input = x_u8_nchw
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.launches = self.run(x_u8_nchw)  # warm: cudaFuncSetAttribute etc.
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.run(x_u8_nchw)
        torch.cuda.synchronize(self.device)
        return self.graph

    def replay(self):
        self.graph.replay()


def make_f32_params(layers: List[ConvLayer], seed: int = 0) -> Dict[str, tuple]:
    """He-normal fp32 weights N(0, sqrt(2 / fan_in)) and biases N(0, 0.01): the
    folded weights and biases of a BN network (w' = w * gain, b' = b * gain +
    shift, folded on the host)."""
    out = {}
    for i, l in enumerate(layers):
        rng = np.random.default_rng([seed, 13, i])
        fan_in = l.cin * l.k * l.k
        w = rng.normal(0.0, np.sqrt(2.0 / fan_in), (l.cout, l.cin, l.k, l.k)).astype(np.float32)
        b = rng.normal(0.0, 0.01, l.cout).astype(np.float32)
        out[l.name] = (w, b)
    return out


def _c16(c: int) -> int:
    return (c + 15) // 16 * 16


class ResNet50F32:
    """fp32 ResNet-50 conv stack on the bf16x3 tensor-core path, resident on
    one GPU: activations stay as split bf16 hi/lo NHWC planes between layers
    (x = hi + lo, the IE_Y_BF16X2_NHWC layout), every conv has its ReLU fused,
    the stem output goes through the 3x3/2 max pool.  ``run(x)`` takes an fp32
    NCHW device tensor [batch, 3, image, image]."""

    def __init__(self, batch: int, params: Dict[str, tuple], device="cuda", image: int = 224):
        import torch

        from . import _lib as L
        self.L, self.torch = L, torch
        self.batch, self.image = batch, image
        self.device = torch.device(device)
        self.layers = resnet50_layers(image)
        dev = self.device
        stream = torch.cuda.current_stream(dev).cuda_stream
        self.descs, self.packed, self.bias, self.acts = {}, {}, {}, {}
        for l in self.layers:
            w, b = params[l.name]
            d = L.ConvDesc()
            d.n, d.c, d.h, d.w, d.m, d.kh, d.kw = batch, l.cin, l.h, l.h, l.cout, l.k, l.k
            d.stride_h = d.stride_w = l.stride
            d.dil_h = d.dil_w = 1
            d.pad_top = d.pad_left = d.pad_bottom = d.pad_right = l.pad
            d.group = 1
            packed = torch.zeros(int(L.lib.ie_cuda_f32_packed_weight_bytes(d)), dtype=torch.uint8,
                                 device=dev)
            L.check(L.lib.ie_cuda_f32_pack_weights(d, torch.from_numpy(w).to(dev).data_ptr(),
                                                   packed.data_ptr(), stream))
            self.descs[l.name], self.packed[l.name] = d, packed
            self.bias[l.name] = torch.from_numpy(b).to(dev)
            self.acts[l.name] = torch.empty((batch, l.out_h, l.out_h, 2 * _c16(l.cout)),
                                            dtype=torch.bfloat16, device=dev)
        self.x_split = torch.empty((batch, image, image, 2 * 16), dtype=torch.bfloat16, device=dev)
        stem = self.layers[0]
        ph = (stem.out_h + 2 - 3) // 2 + 1
        self.acts["pool"] = torch.empty((batch, ph, ph, 2 * 64), dtype=torch.bfloat16, device=dev)
        self.graph = None
        torch.cuda.synchronize(dev)

    @property
    def output(self):
        return self.acts[self.layers[-1].name]

    def to_nchw_f32(self, name: str):
        """A layer's output (or "pool") as fp32 NCHW, hi + lo, on the device."""
        t = self.acts[name]
        half = t.shape[3] // 2
        cout = 64 if name == "pool" else next(l.cout for l in self.layers if l.name == name)
        v = t[..., :half].float() + t[..., half:].float()
        return v[..., :cout].permute(0, 3, 1, 2).contiguous()

    def run(self, x_f32_nchw) -> int:
        L = self.L
        stream = self.torch.cuda.current_stream(self.device).cuda_stream
        b, img = self.batch, self.image
        L.check(L.lib.ie_cuda_f32_pack_input(x_f32_nchw.data_ptr(), self.x_split.data_ptr(), b, 3,
                                             img, img, 16, stream))
        n = 1
        for l in self.layers:
            src = self.x_split if l.src == "input" else self.acts[l.src]
            L.check(L.lib.ie_cuda_conv2d_bf16x3(self.descs[l.name], L.IE_ACT_RELU, src.data_ptr(),
                                                self.packed[l.name].data_ptr(),
                                                self.bias[l.name].data_ptr(),
                                                self.acts[l.name].data_ptr(), L.IE_Y_BF16X2_NHWC,
                                                stream))
            n += 1
            if l.name == "stem":
                s = self.acts["stem"]
                L.check(L.lib.ie_cuda_f32x2_maxpool2d(s.data_ptr(), self.acts["pool"].data_ptr(), b,
                                                      s.shape[1], s.shape[2], 64, 3, 2, 1, stream))
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


def bench_f32(batch: int = 32, iters: int = 20) -> dict:
    """Times the fp32 (bf16x3) stack from a CUDA graph with inputs resident;
    FLOPs are the algorithmic fp32 ones (2 per MAC, stem as the real 7x7x3)."""
    import torch
    layers = resnet50_layers()
    net = ResNet50F32(batch, make_f32_params(layers))
    rng = np.random.default_rng(0)
    x = torch.from_numpy(rng.uniform(-1, 1, (batch, 3, 224, 224)).astype(np.float32)).cuda()
    net.capture(x)
    for _ in range(3):
        net.graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        net.graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    flops = 2 * macs_per_image(layers) * batch
    return {"workload": "ResNet-50 v1.5 fp32 conv stack on bf16x3 (53 convs + max pool)",
            "batch": batch, "ms_per_step": ms, "tflops": flops / ms / 1e9,
            "images_per_s": batch / ms * 1e3, "launches": net.launches,
            "device_error": net.L.take_device_error()}


def main():
    """Runs the int8 stack `--steps` times on cuda:0 (uncaptured launches, so a
    profiler sees each kernel with its own name) and prints one JSON line;
    `--dtype f32` times the fp32 (bf16x3) stack instead."""
    import argparse
    import json

    import torch
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--dtype", choices=["int8", "f32"], default="int8")
    a = ap.parse_args()
    if a.dtype == "f32":
        print(json.dumps(bench_f32(a.batch, max(a.steps, 5))))
        return
    layers = resnet50_layers()
    net = ResNet50Q8(a.batch, make_q8_params(layers))
    x = torch.from_numpy(make_input_u8(a.batch)).cuda()
    launches = 0
    for _ in range(a.steps):
        launches += net.run(x)
    torch.cuda.synchronize()
    print(json.dumps({"batch": a.batch, "steps": a.steps, "launches": launches,
                      "device_error": net.L.take_device_error()}))


if __name__ == "__main__":
    main()
