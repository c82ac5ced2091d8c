#!/usr/bin/env python3
"""Benchmark: int8 ResNet-50 conv stack (53 convolutions) on B200, batch 256
per GPU, batch-sharded across N GPUs (weak scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = the whole stack over one batch of 256 uint8 224x224 images
(stem space-to-depth pack, 53 implicit-GEMM convolutions with fused
requantize, one max pool), replayed from a CUDA graph with the inputs resident
in HBM.  ``value`` is whole-job int8 TOPS (2 ops per MAC, 8.174 GOP per image
counted on the real 7x7 stem); ``e2e`` is the same metric through the C ABI
with host buffers: every step's pinned H2D of its input and D2H of its output
are inside the timed region, on a second stream and double-buffered so that
they overlap the neighbouring steps' compute; with N > 1 each rank first binds
to the CPUs of its GPU's NUMA node so that its pinned buffers live there.  The
working set (5.6 GB of activations per step) is far larger than L2, so no
flush is needed between steps.

``--impl reference`` times the reference engine's own CPU convolution
(Conv2DOp compiled from its sources, fp32, run on the dequantized stack, one
image per host thread) on a bounded sample of the same workload: each step is
a window of consecutive layers, rotating through the stack, sized so that all
K steps take about REFERENCE_ARM_BUDGET_S of host time.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BATCH_PER_GPU = 256
IMAGE = 224
PROFILE_JSON = ROOT / "profiles" / "conv_igemm_q8_resnet50_traffic.json"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=BATCH_PER_GPU)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.skip = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # nvidia-smi takes a few hundred ms to print its first line: wait for
            # it so that the samples fall inside the timed region that follows.
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0:
                time.sleep(0.01)
            self.skip = len(self.lines)
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = self.lines[self.skip:]
        note = None
        if not lines and self.lines:
            # the timed region ended before the next sample: report the one
            # taken as it started (the warm-up had the GPU busy then)
            lines, note = self.lines[-1:], "timed region shorter than the sampling period"
        for ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        out = {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
               "samples": len(sm)}
        if note:
            out["note"] = note
        return out


# ------------------------------------------------------------ distributed

def dist_setup(want_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# -------------------------------------------------------- CPU reference arm

def _dequant_stack(layers, params):
    """fp32 weights / biases of the dequantized stack for the reference conv."""
    out = {}
    for l in layers:
        p = params[l.name]
        s_w = p.s_w.astype(np.float32)
        w = p.w.astype(np.float32) * s_w.reshape(-1, 1, 1, 1)
        b = p.bias.astype(np.float32) * (np.float32(p.s_x) * s_w)
        out[l.name] = (np.ascontiguousarray(w), b)
    return out


def cpu_reference_stack(images: int, threads: int):
    """Runs the reference's fp32 Conv2DOp over the 53-layer stack on `images`
    images (one op call per image per thread).  Returns (seconds, kind, cores,
    row_kernel)."""
    from computeengine_b200.resnet import make_input_u8, make_q8_params, resnet50_layers
    from oracle.oracle import Oracle, RefConv, maxpool2d_nchw

    layers = resnet50_layers(IMAGE)
    params = make_q8_params(layers, seed=0)
    x = make_input_u8(images, seed=123)
    if RefConv.available():
        ref = RefConv()
        fp = _dequant_stack(layers, params)
        xf = (x.astype(np.float32) - 128.0) * np.float32(0.02)
        acts = {}
        last_use = {}
        for i, l in enumerate(layers):
            last_use[l.src] = i
        t0 = time.perf_counter()
        for i, l in enumerate(layers):
            src = xf if l.src == "input" else acts[l.src]
            w, b = fp[l.name]
            rc, y = ref.conv2d(src, w, b, strides=(l.stride, l.stride), pads=(l.pad,) * 4,
                               nthreads=threads)
            if rc != 0:
                raise RuntimeError(f"reference conv failed on {l.name}: {rc}")
            np.maximum(y, 0.0, out=y)
            acts[l.name] = y
            if l.name == "stem":
                acts["pool"] = maxpool2d_nchw(y, 3, 2, 1)
            for name in [k for k in acts if last_use.get(k, -1) <= i]:
                del acts[name]  # dead tensors: keeps host memory to two blocks' worth
        return time.perf_counter() - t0, "reference", threads, ref.row_kernel()
    orc = Oracle()
    outs = {}
    t0 = time.perf_counter()
    for l in layers:
        p = params[l.name]
        src = x if l.src == "input" else outs[l.src]
        outs[l.name] = orc.conv2d_q8(src, p.w, p.bias, p.mult, p.zp_x, 0, 0, 255,
                                     strides=(l.stride, l.stride), pads=(l.pad,) * 4,
                                     nthreads=threads)
        if l.name == "stem":
            outs["pool"] = maxpool2d_nchw(outs["stem"], 3, 2, 1)
    return time.perf_counter() - t0, "port", threads, "c-oracle"


def cpu_threads() -> int:
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    return max(1, min(n, 32))


def cpu_model() -> str:
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class CpuLayerRunner:
    """The stack's convolutions run one layer at a time on the host cores: the
    reference's fp32 Conv2DOp on the dequantized stack when its library is
    built, else the int8 oracle port.  Each layer reads a fixed synthetic input
    of its own shape (`images` images, one per thread), so any contiguous
    window of layers can be timed on its own; a dense convolution's time does
    not depend on its values."""

    def __init__(self, images: int, threads: int):
        from computeengine_b200.resnet import make_q8_params, resnet50_layers
        from oracle.oracle import Oracle, RefConv

        self.layers = resnet50_layers(IMAGE)
        self.params = make_q8_params(self.layers, seed=0)
        self.images, self.threads = images, threads
        rng = np.random.default_rng(7)
        self.inputs = {}
        if RefConv.available():
            self.kind, self.ref = "reference", RefConv()
            self.row_kernel = self.ref.row_kernel()
            self.fp = _dequant_stack(self.layers, self.params)
            for l in self.layers:
                key = (l.cin, l.h)
                if key not in self.inputs:
                    x = rng.integers(0, 40, (images, l.cin, l.h, l.h), dtype=np.uint8)
                    self.inputs[key] = x.astype(np.float32) * np.float32(0.05)
        else:
            self.kind, self.orc, self.row_kernel = "port", Oracle(), "c-oracle"
            for l in self.layers:
                key = (l.cin, l.h)
                if key not in self.inputs:
                    self.inputs[key] = rng.integers(0, 40, (images, l.cin, l.h, l.h),
                                                    dtype=np.uint8)

    def run_layer(self, i: int) -> float:
        """Runs layer i on its synthetic input; returns seconds."""
        l = self.layers[i]
        x = self.inputs[(l.cin, l.h)]
        t0 = time.perf_counter()
        if self.kind == "reference":
            w, b = self.fp[l.name]
            rc, y = self.ref.conv2d(x, w, b, strides=(l.stride, l.stride), pads=(l.pad,) * 4,
                                    nthreads=self.threads)
            if rc != 0:
                raise RuntimeError(f"reference conv failed on {l.name}: {rc}")
            np.maximum(y, 0.0, out=y)
        else:
            p = self.params[l.name]
            self.orc.conv2d_q8(x, p.w, p.bias, p.mult, p.zp_x, 0, 0, 255,
                               strides=(l.stride, l.stride), pads=(l.pad,) * 4,
                               nthreads=self.threads)
        return time.perf_counter() - t0


# Host seconds the reference arm's timed steps may take in total, whatever K is.
REFERENCE_ARM_BUDGET_S = 150.0


def run_reference_arm(args, world, rank):
    """The reference's CPU path timed over K steps.  A full step (53 convs on one
    image per host thread) takes several seconds, so each step is a window of
    consecutive layers sized from an untimed calibration pass to keep all K
    steps within REFERENCE_ARM_BUDGET_S; the windows rotate through the stack,
    and the value is the operations done over the time taken.  With K small
    enough every step is the whole stack."""
    if rank != 0:
        return
    threads = cpu_threads()
    images = threads
    runner = CpuLayerRunner(images, threads)
    nl = len(runner.layers)
    layer_ops = [2 * l.macs_per_image * images for l in runner.layers]
    calib = [runner.run_layer(i) for i in range(nl)]  # untimed: page-in, thread start-up
    step_budget = min(sum(calib), REFERENCE_ARM_BUDGET_S / max(args.steps, 1))
    for _ in range(args.warmup):
        runner.run_layer(0)
    cursor, tot, ops, layers_run = 0, 0.0, 0, 0
    for _ in range(args.steps):
        est, window = 0.0, []
        while len(window) < nl and (not window or est + calib[cursor] <= step_budget * 1.05):
            window.append(cursor)
            est += calib[cursor]
            cursor = (cursor + 1) % nl
        for i in window:
            tot += runner.run_layer(i)
            ops += layer_ops[i]
        layers_run += len(window)
    value = ops / tot / 1e12
    sample = (f"{images} images (one per host thread); {layers_run} layer runs over "
              f"{args.steps} steps, rotating through the 53 convs "
              f"({layers_run / nl:.2f} passes of the stack)")
    line = {
        "metric": "int8 conv TOPS (ResNet-50 conv stack, 53 convs)",
        "value": value, "unit": "TOPS", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": tot / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32" if runner.kind == "reference" else "int8",
        "data": "synthetic (seeded)",
        "images_per_s": value * 1e12 / sum(layer_ops) * images,
        "config": {"workload": "ResNet-50 v1.5 conv stack, reference Conv2DOp on the "
                               "dequantized int8 stack (fp32), one image per host thread",
                   "batch_per_step": images, "image": IMAGE, "row_kernel": runner.row_kernel,
                   "cpu": cpu_model()},
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": threads, "kind": runner.kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ ours

def run_ours(args, world, rank, local):
    import torch

    from computeengine_b200 import _lib as L
    from computeengine_b200.resnet import (ResNet50Q8, macs_per_image, make_input_u8,
                                           make_q8_params, resnet50_layers)
    from computeengine_b200.shard import (bind_to_pci_local_cpus, broadcast_from_rank0,
                                          input_seed, max_over_ranks, shard_batch)

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    prev_affinity = None
    if world > 1:
        # every rank's pinned input and output buffers on its GPU's NUMA node
        props = torch.cuda.get_device_properties(dev)
        prev_affinity = bind_to_pci_local_cpus(props.pci_domain_id, props.pci_bus_id,
                                               props.pci_device_id)
    layers = resnet50_layers(IMAGE)
    ops_img = 2 * macs_per_image(layers)
    b = args.batch
    params = make_q8_params(layers, seed=0)
    net = ResNet50Q8(b, params, device=dev)
    # weights, biases and multipliers go out once from rank 0 (NCCL over NVLink)
    broadcast_bytes = broadcast_from_rank0(net.tensors())
    torch.cuda.synchronize(dev)

    first, count = shard_batch(b * world, world, rank)
    assert count == b
    x_host = make_input_u8(b, seed=input_seed(0, rank))
    x_pin = torch.from_numpy(x_host).pin_memory()
    x_dev = x_pin.to(dev)
    net.capture(x_dev)
    per_step_launches = net.launches

    # ---- device-resident throughput (the `value`)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        net.replay()
    torch.cuda.synchronize(dev)
    barrier(world)
    L.launch_count(reset=True)
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize(dev)
        start.record(stream)
        for _ in range(args.steps):
            net.replay()
        stop.record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
    ms = start.elapsed_time(stop)
    ms_max = max_over_ranks(ms, dev)
    assert L.take_device_error() == 0, "a kernel reported a bounded-wait timeout"
    total_images = b * world * args.steps
    value = ops_img * total_images / (ms_max / 1e3) / 1e12

    # ---- per-kernel durations of the convolutions (roofline of the dominant kernel)
    conv_ms, conv_ops = per_layer_times(net, layers, x_dev, args.steps, ops_img // 2, b)

    # ---- end to end through the C ABI with host buffers: every step copies its
    # input from pinned host memory and reads its output back; the copies run
    # on a second stream, double-buffered, so that step i+1's upload and step
    # i-1's download overlap step i's compute (as a serving loop would)
    copy = torch.cuda.Stream(dev)
    x_next = torch.empty_like(x_dev)
    out_stage = [torch.empty_like(net.output) for _ in range(2)]
    out_pin = [torch.empty(net.output.shape, dtype=torch.uint8).pin_memory() for _ in range(2)]

    def e2e_steps(nsteps):
        d2h_done = [None, None]
        with torch.cuda.stream(copy):
            x_next.copy_(x_pin, non_blocking=True)
        h2d_done = copy.record_event()
        for i in range(nsteps):
            stream.wait_event(h2d_done)
            x_dev.copy_(x_next, non_blocking=True)
            x_free = stream.record_event()
            if i + 1 < nsteps:
                copy.wait_event(x_free)
                with torch.cuda.stream(copy):
                    x_next.copy_(x_pin, non_blocking=True)
                h2d_done = copy.record_event()
            net.replay()
            j = i % 2
            if d2h_done[j] is not None:
                stream.wait_event(d2h_done[j])
            out_stage[j].copy_(net.output, non_blocking=True)
            copy.wait_event(stream.record_event())
            with torch.cuda.stream(copy):
                out_pin[j].copy_(out_stage[j], non_blocking=True)
            d2h_done[j] = copy.record_event()
        stream.wait_stream(copy)

    e2e_steps(2)
    torch.cuda.synchronize(dev)
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), dev)
    e2e_value = ops_img * total_images / (e2e_ms / 1e3) / 1e12

    if prev_affinity is not None:
        os.sched_setaffinity(0, prev_affinity)

    # ---- CPU baseline (rank 0, single GPU runs only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = cpu_threads()
        cpu_reference_stack(1, 1)  # untimed: page-in, thread start-up
        dt, passes = 0.0, 0
        while dt < 10.0 and passes < 30:  # about 10 s of host work
            t, kind, cores, rk = cpu_reference_stack(threads, threads)
            dt += t
            passes += 1
        cpu = {"value": ops_img * threads * passes / dt / 1e12, "unit": "TOPS", "cores": cores,
               "kind": kind,
               "sample": f"{passes} passes of {threads} images through the 53-conv stack, "
                         f"one image per thread ({rk} row kernel, {cpu_model()})",
               "images_per_s": threads * passes / dt}

    if rank != 0:
        return
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    bf16 = peaks.get("bf16_tflops")
    peak_src = "2x measured cuBLAS bf16 burst (MEASURED_PEAKS.json)"
    if bf16 is None:
        bf16, peak_src = 1590.0, "2x fallback bf16 1.59 PFLOP/s"
    peak = 2.0 * bf16
    achieved = conv_ops * 2 / (conv_ms / 1e3) / 1e12  # TOPS over the conv launches
    traffic = None
    if PROFILE_JSON.exists():
        prof = json.loads(PROFILE_JSON.read_text())
        if prof.get("batch") == b:
            traffic = prof.get("dram_bytes_per_launch")
    line = {
        "metric": "int8 conv TOPS (ResNet-50 conv stack, 53 convs)",
        "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded uint8 images, seeded int8 weights)",
        "images_per_s": total_images / (ms_max / 1e3),
        "frac_of_nominal_int8_4500": value / world / 4500.0,
        "config": {"workload": "ResNet-50 v1.5 int8 conv stack (53 convs + stem pack + maxpool), "
                               "CUDA-graph replay",
                   "global_batch": b * world, "batch_per_gpu": b, "image": IMAGE,
                   "parallelism": f"batch-sharded dp{world}, weights broadcast once "
                                  f"({broadcast_bytes} bytes)",
                   "l2": "working set 5.6 GB/step >> 126 MB L2, no flush"},
        "gpu_launches": per_step_launches * args.steps,
        "e2e": {"value": e2e_value, "unit": "TOPS",
                "h2d_bytes_per_step": int(x_pin.numel()),
                "d2h_bytes_per_step": int(out_pin[0].numel()),
                "copies": "pinned H2D / D2H on a second stream, double-buffered"},
        "roofline": {"bound": "tensor", "kernel": "conv_igemm_kernel (int8, all 53 layers)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": peak_src,
                     "traffic": traffic,
                     "conv_ms_per_step": conv_ms, "step_ms": ms_max / args.steps},
        "clocks": clocks.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def per_layer_times(net, layers, x_dev, steps, macs_img, batch):
    """Times every convolution launch with external CUDA events captured into a
    second graph of the stack; returns (ms of all conv launches per step,
    MACs per step)."""
    import torch
    L = net.L
    dev = net.device
    stream_handle = None
    evs = []
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            stream_handle = torch.cuda.current_stream(dev).cuda_stream
            cur = torch.cuda.current_stream(dev)
            L.check(L.lib.ie_cuda_q8_stem_pack_input(x_dev.data_ptr(), net.stem_in.data_ptr(),
                                                     net.batch, 3, net.image, net.image, 0x80,
                                                     stream_handle))
            for l in layers:
                src = net.stem_in if l.src == "input" else net.acts[l.src]
                a = torch.cuda.Event(enable_timing=True, external=True)
                z = torch.cuda.Event(enable_timing=True, external=True)
                a.record(cur)
                L.check(L.lib.ie_cuda_conv2d_q8(net.descs[l.name], net.qp[l.name], src.data_ptr(),
                                                net.packed[l.name].data_ptr(),
                                                net.bias[l.name].data_ptr(),
                                                net.mult[l.name].data_ptr(),
                                                net.acts[l.name].data_ptr(), stream_handle))
                z.record(cur)
                evs.append((l, a, z))
                if l.name == "stem":
                    st = net.acts["stem"]
                    L.check(L.lib.ie_cuda_q8_maxpool2d(st.data_ptr(), net.acts["pool"].data_ptr(),
                                                       net.batch, st.shape[1], st.shape[2], 64, 3,
                                                       2, 1, 0, stream_handle))
    torch.cuda.synchronize(dev)
    tot = {l.name: 0.0 for l in layers}
    reps = max(3, min(steps, 10))
    for _ in range(reps):
        g.replay()
        torch.cuda.synchronize(dev)
        for l, a, z in evs:
            tot[l.name] += a.elapsed_time(z)
    conv_ms = sum(tot.values()) / reps
    net.layer_ms = {k: v / reps for k, v in tot.items()}
    return conv_ms, macs_img * batch


def main():
    args = parse_args()
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference_arm(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
