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
import ctypes
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
    ap.add_argument("--no-workloads", action="store_true",
                    help="skip the single-conv, fp32-stack and MobileNetV2 workloads")
    return ap.parse_args()


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """Samples the GPU's SM clock, board power and clock-event (throttle)
    reasons while the timed region runs.  Read-only NVML queries every 5 ms,
    so even a timed region of a few tens of milliseconds gets several samples;
    nvidia-smi every 100 ms when NVML is unavailable.  mark_start() /
    mark_stop() bracket the timed region on the host clock: only samples taken
    between them are summarised."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, pci_bus_id: str = None, period_s: float = 0.005):
        self.gpu, self.pci, self.period = gpu_index, pci_bus_id, period_s
        self.samples = []  # (host time, sm MHz, power W, [reason names])
        self.max_mhz = None
        self.source = None
        self.t0 = self.t1 = None
        self._stop = threading.Event()
        self._thread = None
        self._proc = None

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_stop(self):
        self.t1 = time.perf_counter()

    def _nvml_loop(self, nv, h):
        masks = [(name, getattr(nv, attr, 0)) for name, attr in self.REASONS]
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((time.perf_counter(), float(sm), pw,
                                     [n for n, m in masks if m and bits & m]))
            except Exception:  # pragma: no cover - a transient NVML error skips a sample
                pass
            self._stop.wait(self.period)

    def _smi_loop(self):
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm, self.max_mhz = float(parts[1]), float(parts[2])
                pw = float(parts[3])
            except ValueError:
                continue
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            self.samples.append((time.perf_counter(), sm, pw,
                                 [n for n, v in zip(names, parts[5:9]) if v.lower() == "active"]))

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = (nv.nvmlDeviceGetHandleByPciBusId(self.pci) if self.pci
                 else nv.nvmlDeviceGetHandleByIndex(self.gpu))
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self._thread = threading.Thread(target=self._nvml_loop, args=(nv, h), daemon=True)
            self.source = "nvml (5 ms)"
        except Exception:
            try:
                self._proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.SMI_FIELDS}",
                     "--format=csv,noheader,nounits", "-lms", "100"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self._thread = threading.Thread(target=self._smi_loop, daemon=True)
                self.source = "nvidia-smi (100 ms)"
            except FileNotFoundError:
                return self
        self._thread.start()
        t0 = time.time()
        while not self.samples and time.time() - t0 < 3.0:  # first sample before timing
            time.sleep(0.002)
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        inside = [s for s in self.samples
                  if (self.t0 is None or s[0] >= self.t0) and (self.t1 is None or s[0] <= self.t1)]
        note = None
        if not inside and self.samples:
            before = [s for s in self.samples if self.t0 is None or s[0] < self.t0]
            inside = before[-1:] or self.samples[:1]
            note = "timed region shorter than the sampling period: the last sample before it"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": self.source}
        reasons = sorted({r for s in inside for r in s[3]})
        out = {"sm_mhz": float(np.median([s[1] for s in inside])),
               "sm_mhz_min": float(min(s[1] for s in inside)), "sm_max_mhz": self.max_mhz,
               "power_w_max": float(max(s[2] for s in inside)), "reasons": reasons,
               "samples": len(inside), "source": self.source}
        if note:
            out["note"] = note
        return out


# ------------------------------------------------------------ distributed

def dist_setup(want_gpus: int, impl: str = "ours"):
    """Rank, world size and local rank from torchrun's environment.  Our arm
    joins an NCCL process group (weights broadcast, barriers, max over ranks);
    the reference arm runs on rank 0's host cores only and touches no GPU, so
    it joins none."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and impl == "ours":
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


# ------------------------------------------------------- the other workloads

def _ref_seconds(fn, min_s=1.0, max_reps=50):
    """Host seconds per call of fn (one untimed call, then repeats for about
    min_s seconds)."""
    fn()
    reps, t0 = 0, time.perf_counter()
    while reps < max_reps and (reps == 0 or time.perf_counter() - t0 < min_s):
        fn()
        reps += 1
    return (time.perf_counter() - t0) / reps


def cpu_workloads(threads: int, stack_tops: float = None) -> dict:
    """The reference's fp32 Conv2DOp (oracle/_ref) on the host cores for the
    single-convolution, fp32-stack and MobileNetV2 workloads; int8 workloads run
    on their dequantized tensors (the reference has no int8 convolution).
    Returns per config {"value", "unit", "cores", "sample"}."""
    from oracle.oracle import RefConv
    if not RefConv.available():
        return {}
    from computeengine_b200.mobilenet import mobilenetv2_layers
    ref = RefConv()
    rng = np.random.default_rng(0)
    out = {}
    # config 1: one fp32 conv + ReLU, one call on one core (the op is single-threaded)
    x = rng.uniform(-1, 1, (1, 64, 56, 56)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2 / 576), (64, 64, 3, 3)).astype(np.float32)
    b = rng.normal(0, 0.01, 64).astype(np.float32)

    def c1():
        rc, y = ref.conv2d(x, w, b, pads=(1, 1, 1, 1))
        np.maximum(y, 0.0, out=y)
    t = _ref_seconds(c1)
    out["1"] = {"value": 2 * 64 * 64 * 9 * 56 * 56 / t / 1e12, "unit": "TFLOP/s", "cores": 1,
                "sample": "reference Conv2DOp + Relu on [1,64,56,56], repeated ~1 s"}
    # config 2: the int8 conv dequantized, one image per thread
    n2 = min(8, threads)
    x2 = rng.normal(0, 0.6, (n2, 128, 28, 28)).astype(np.float32)
    w2 = rng.normal(0, 0.3, (128, 128, 3, 3)).astype(np.float32)
    t = _ref_seconds(lambda: ref.conv2d(x2, w2, None, pads=(1, 1, 1, 1), nthreads=n2))
    out["2"] = {"value": n2 * 2 * 128 * 128 * 9 * 28 * 28 / t / 1e12, "unit": "TOPS",
                "cores": n2, "sample": f"reference Conv2DOp (fp32) on the dequantized "
                                       f"[{n2},128,28,28] conv, one image per thread"}
    # config 3: the fp32 stack's ops per image equal the int8 stack's; the
    # reference stack measured for the headline's cpu_baseline is this one
    if stack_tops is not None:
        out["3"] = {"value": stack_tops, "unit": "TFLOP/s", "cores": threads,
                    "sample": "the reference fp32 Conv2DOp ResNet-50 stack timed for the headline "
                              "cpu_baseline (same convolutions, same FLOPs per image)"}
    # config 4: the MobileNetV2 sweep, fp32 on dequantized tensors, one image per thread
    layers = mobilenetv2_layers()
    xs = {}
    for l in layers:
        key = (l.cin, l.h)
        if key not in xs:
            xs[key] = rng.uniform(0, 2, (threads, l.cin, l.h, l.h)).astype(np.float32)
    ws = [rng.normal(0, 0.1, (l.cout, 1 if l.kind == "dw" else l.cin, l.k, l.k)).astype(np.float32)
          for l in layers]

    def c4():
        for l, wl in zip(layers, ws):
            g = l.cin if l.kind == "dw" else 1
            ref.conv2d(xs[(l.cin, l.h)], wl, None, strides=(l.stride, l.stride),
                       pads=(l.k // 2,) * 4, group=g, depthwise=l.kind == "dw", nthreads=threads)
    t = _ref_seconds(c4, min_s=2.0, max_reps=5)
    macs = sum(l.macs_per_image for l in layers)
    out["4"] = {"value": threads * 2 * macs / t / 1e12, "unit": "TOPS", "cores": threads,
                "images_per_s": threads / t,
                "sample": f"reference Conv2DOp / DepthwiseConv2DOp (fp32) over the 17-block "
                          f"sweep's 52 convolutions, {threads} images, one per thread"}
    return out


def engine_resnet50_q8(batch: int = 256, iters: int = 20, warmup: int = 3) -> dict:
    """The int8 ResNet-50 as one engine graph (the 53 convolutions, the max
    pool, the 16 int8 shortcut Adds, the int8 GAP, the FC) run through the C++
    CudaExecutor -- the reference Executor's interface -- with host tensors in
    and out: per run the pinned upload of the uint8 batch, every node launched
    from its op's forward(), the logits downloaded, one synchronize.  Timed by
    the host clock around the synchronous calls in the backend's test driver
    (a separate process on the same GPU); its check that one image alone gives
    the batch's first row of logits is part of the line."""
    from computeengine_b200.build import BACKEND_TEST, build
    try:
        if not BACKEND_TEST.exists():
            build()
        out = subprocess.run([str(BACKEND_TEST), "engine-bench", str(batch), str(iters), str(warmup)],
                             capture_output=True, text=True, timeout=600)
    except (OSError, RuntimeError, subprocess.SubprocessError) as e:
        return {"error": f"engine-bench did not run: {e}"}
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    r = json.loads(lines[-1]) if lines else {"error": (out.stderr or out.stdout)[-300:]}
    r["returncode"] = out.returncode
    r["workload"] = ("int8 ResNet-50 graph (53 convs, max pool, 16 int8 Adds, GAP, FC) through "
                     "CudaExecutor::run, host tensors in and out")
    return r


def gpu_workloads(peaks: dict) -> dict:
    """Configs 1-4 on this GPU (CUDA events on the launching stream, after
    warm-up), each with its roofline fraction and the denominator it uses."""
    from computeengine_b200 import conv_bench, mobilenet, resnet
    bf16 = peaks.get("bf16_tflops", 1590.0)
    hbm = peaks.get("hbm_gbs", 6650.0)
    src = "MEASURED_PEAKS.json" if "bf16_tflops" in peaks else "fallback"
    c12 = {r["config"]: r for r in conv_bench.bench_configs(iters=200)}
    r1, r2 = c12[1], c12[2]
    f3 = resnet.bench_f32(32, iters=20)
    m4 = mobilenet.benchmark(64, 50)
    engine = engine_resnet50_q8()
    return {
        "engine": engine,
        "1": {"workload": r1["workload"], "value": r1["gflops"] / 1e3, "unit": "TFLOP/s",
              "us_per_call": r1["us"], "dtype": "f32 (bf16x3)",
              "e2e": {"value": 2 * 64 * 64 * 9 * 56 * 56 / r1["e2e_us"] / 1e6, "unit": "TFLOP/s",
                      "us_per_call": r1["e2e_us"], "how": r1["e2e"]},
              "roofline": {"bound": "latency (0.23 GFLOP, three launches)",
                           "frac": r1["frac_of_bf16_peak_over_3"],
                           "denominator": f"bf16 burst / 3 = {bf16 / 3:.0f} TFLOP/s ({src})"}},
        "2": {"workload": r2["workload"], "value": r2["kernel_tops"], "unit": "TOPS",
              "kernel_us": r2["kernel_us"], "drop_in_us": r2["drop_in_us"],
              "drop_in_tops": r2["drop_in_tops"], "dtype": "int8",
              "e2e": {"value": 2 * 8 * 128 * 128 * 9 * 28 * 28 / r2["e2e_us"] / 1e6, "unit": "TOPS",
                      "us_per_call": r2["e2e_us"], "how": r2["e2e"]},
              "roofline": {"bound": "tensor", "frac": r2["frac_of_2x_bf16_peak"],
                           "denominator": f"2 x bf16 burst = {2 * bf16:.0f} TOPS ({src})"}},
        "3": {"workload": f3["workload"], "value": f3["tflops"], "unit": "TFLOP/s",
              "ms_per_step": f3["ms_per_step"], "batch": f3["batch"],
              "images_per_s": f3["images_per_s"], "dtype": "f32 (bf16x3)",
              "roofline": {"bound": "tensor", "frac": f3["tflops"] / (bf16 / 3),
                           "denominator": f"bf16 burst / 3 = {bf16 / 3:.0f} TFLOP/s ({src})"}},
        "4": {"workload": m4["workload"], "value": m4["tops"], "unit": "TOPS",
              "ms_per_step": m4["ms_per_step"], "batch": m4["batch"],
              "images_per_s": m4["images_per_s"], "dtype": "int8",
              "algorithmic_gbs": m4["algorithmic_gbs"],
              "roofline": {"bound": "hbm", "frac": m4["algorithmic_gbs"] / hbm,
                           "denominator": f"HBM copy {hbm:.0f} GB/s ({src})"}},
    }


# ------------------------------------------------------------------ ours

def run_ours(args, world, rank, local):
    import torch

    from computeengine_b200 import _lib as L
    from computeengine_b200.resnet import (ResNet50Q8, macs_per_image, make_input_u8,
                                           make_q8_params, resnet50_layers)
    from computeengine_b200.shard import (bind_to_pci_local_cpus, broadcast_from_rank0_checked,
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
    ok, msg, broadcast_bytes = broadcast_from_rank0_checked(net.tensors())
    if not ok:
        raise SystemExit(f"rank {rank}: weight broadcast failed: {msg}")
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
    props = torch.cuda.get_device_properties(dev)
    pci = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    with ClockSampler(local, pci) as clocks:
        barrier(world)
        torch.cuda.synchronize(dev)
        clocks.mark_start()
        start.record(stream)
        for _ in range(args.steps):
            net.replay()
        stop.record(stream)
        torch.cuda.synchronize(dev)
        clocks.mark_stop()
        barrier(world)
    ms = start.elapsed_time(stop)
    ms_max = max_over_ranks(ms, dev)
    assert L.take_device_error() == 0, "a kernel reported a bounded-wait timeout"
    total_images = b * world * args.steps
    value = ops_img * total_images / (ms_max / 1e3) / 1e12

    # ---- per-launch durations of the convolutions (roofline of the dominant kernel)
    conv_ms, conv_ops = per_layer_times(net, layers, ops_img // 2, b)

    # ---- end to end through the C ABI with host buffers: every step copies its
    # input from pinned host memory and reads its output back; uploads and
    # downloads run on two copy streams of their own (the link carries both
    # directions at once), double-buffered, so that step i+1's upload and step
    # i-1's download overlap step i's compute (as a serving loop would)
    up = torch.cuda.Stream(dev)
    down = torch.cuda.Stream(dev)
    x_next = torch.empty_like(x_dev)
    out_stage = [torch.empty_like(net.output) for _ in range(2)]
    out_pin = [torch.empty(net.output.shape, dtype=torch.uint8).pin_memory() for _ in range(2)]

    def e2e_steps(nsteps, compute=True):
        d2h_done = [None, None]
        with torch.cuda.stream(up):
            x_next.copy_(x_pin, non_blocking=True)
        h2d_done = up.record_event()
        for i in range(nsteps):
            stream.wait_event(h2d_done)
            x_dev.copy_(x_next, non_blocking=True)
            x_free = stream.record_event()
            if i + 1 < nsteps:
                up.wait_event(x_free)
                with torch.cuda.stream(up):
                    x_next.copy_(x_pin, non_blocking=True)
                h2d_done = up.record_event()
            if compute:
                net.replay()
            j = i % 2
            if d2h_done[j] is not None:
                stream.wait_event(d2h_done[j])
            out_stage[j].copy_(net.output, non_blocking=True)
            down.wait_event(stream.record_event())
            with torch.cuda.stream(down):
                out_pin[j].copy_(out_stage[j], non_blocking=True)
            d2h_done[j] = down.record_event()
        stream.wait_stream(up)
        stream.wait_stream(down)

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
    # the same loop with the stack left out: the pinned-copy ceiling of e2e on
    # this box (all ranks copy at once, as in the e2e run)
    e2e_steps(2, compute=False)
    torch.cuda.synchronize(dev)
    barrier(world)
    e0.record(stream)
    e2e_steps(args.steps, compute=False)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    copy_ms = max_over_ranks(e0.elapsed_time(e1), dev)
    copy_value = ops_img * total_images / (copy_ms / 1e3) / 1e12

    if prev_affinity is not None:
        os.sched_setaffinity(0, prev_affinity)

    # ---- CPU baseline (rank 0, single GPU runs only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = cpu_threads()
        cpu_reference_stack(1, 1)  # untimed: page-in, thread start-up
        t1, _, _, _ = cpu_reference_stack(1, 1)  # one image on one thread
        dt, passes = 0.0, 0
        while dt < 10.0 and passes < 30:  # about 10 s of host work
            t, kind, cores, rk = cpu_reference_stack(threads, threads)
            dt += t
            passes += 1
        cpu = {"value": ops_img * threads * passes / dt / 1e12, "unit": "TOPS", "cores": cores,
               "kind": kind,
               "sample": f"{passes} passes of {threads} images through the 53-conv stack, "
                         f"one image per thread ({rk} row kernel, {cpu_model()})",
               "images_per_s": threads * passes / dt,
               "single_thread": {"value": ops_img / t1 / 1e12, "unit": "TOPS",
                                 "images_per_s": 1.0 / t1},
               "host_threads": os.cpu_count(), "cpu_model": cpu_model()}

    if rank != 0:
        return
    # this GPU's own int8 tensor-core rate (back-to-back tcgen05.mma kind::i8,
    # M=128 N=256 K=32, every SM), after every timed region
    i8_peak = ctypes.c_double()
    L.check(L.lib.ie_cuda_mma_i8_peak(40000, ctypes.byref(i8_peak),
                                      torch.cuda.current_stream(dev).cuda_stream))
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    workloads = None
    if world == 1 and not args.no_workloads:
        workloads = gpu_workloads(peaks)
        if cpu is not None:
            for k, v in cpu_workloads(cpu_threads(), cpu["value"]).items():
                workloads[k]["cpu_baseline"] = v
    bf16 = peaks.get("bf16_tflops")
    peak_src = "2x measured cuBLAS bf16 burst (MEASURED_PEAKS.json)"
    if bf16 is None:
        bf16, peak_src = 1590.0, "2x fallback bf16 1.59 PFLOP/s"
    peak = 2.0 * bf16
    achieved = conv_ops * 2 / (conv_ms / 1e3) / 1e12  # TOPS over the conv launches
    step_ms = ms_max / args.steps
    traffic = None
    traffic_note = None
    if PROFILE_JSON.exists():
        prof = json.loads(PROFILE_JSON.read_text())
        if prof.get("scale_to_batch", prof.get("batch")) == b:
            traffic = prof.get("dram_bytes_per_launch")
            traffic_note = prof.get("note")
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
                "copies": "pinned H2D and D2H on two copy streams (both link directions at once), double-buffered",
                "copy_only_ms_per_step": copy_ms / args.steps,
                "copy_only_ceiling": copy_value,
                "frac_of_copy_ceiling": e2e_value / copy_value,
                "host_copy_gbs": (int(x_pin.numel()) + int(out_pin[0].numel())) * world
                                 * args.steps / (copy_ms / 1e3) / 1e9},
        "roofline": {"bound": "tensor", "kernel": "conv_igemm_kernel (int8, all 53 layers)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": peak_src,
                     "traffic": traffic, "traffic_note": traffic_note,
                     "conv_ms_per_step": conv_ms, "step_ms": step_ms,
                     "conv_share_of_step": conv_ms / step_ms,
                     "timing": "each conv launch timed in a CUDA graph of 10 back-to-back "
                               "launches of itself (events on the replay stream); achieved = "
                               "ops of the 53 convs / the sum of their launch times",
                     "frac_of_nominal_int8_4500": achieved / 4500.0,
                     "measured_int8_peak": i8_peak.value,
                     "frac_of_measured_int8_peak": achieved / i8_peak.value,
                     "measured_int8_peak_source": "ie_cuda_mma_i8_peak: 40000 back-to-back "
                                                  "tcgen05.mma kind::i8 M=128 N=256 K=32 per "
                                                  "SM, this GPU, this run",
                     "layer_us": {k: round(v * 1e3, 2) for k, v in net.layer_ms.items()}},
        "clocks": clocks.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if workloads is not None:
        line["workloads"] = workloads
    print(json.dumps(line), flush=True)


def per_layer_times(net, layers, macs_img, batch, reps=10):
    """Per-launch durations of the 53 convolutions in the regime the step runs
    in: each layer's launch is captured `reps` times back to back into a CUDA
    graph of its own, replayed once to warm, then timed with CUDA events on the
    replay stream.  Returns (ms of one launch of every conv, summed; MACs per
    step).  Unlike events recorded between the kernels of the step's graph,
    this adds no event node between launches, so the sum can be compared with
    the step time."""
    import torch
    L = net.L
    dev = net.device
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    torch.cuda.synchronize(dev)
    per = {}
    for l in layers:
        src = net.stem_in if l.src == "input" else net.acts[l.src]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                h = torch.cuda.current_stream(dev).cuda_stream
                for _ in range(reps):
                    L.check(L.lib.ie_cuda_conv2d_q8(net.descs[l.name], net.qp[l.name],
                                                    src.data_ptr(), net.packed[l.name].data_ptr(),
                                                    net.bias[l.name].data_ptr(),
                                                    net.mult[l.name].data_ptr(),
                                                    net.acts[l.name].data_ptr(), h))
        with torch.cuda.stream(s):
            g.replay()
            a = torch.cuda.Event(enable_timing=True)
            z = torch.cuda.Event(enable_timing=True)
            a.record(s)
            g.replay()
            z.record(s)
        torch.cuda.synchronize(dev)
        per[l.name] = a.elapsed_time(z) / reps
        del g
    net.layer_ms = per
    return sum(per.values()), macs_img * batch


def main():
    args = parse_args()
    world, rank, local = dist_setup(args.gpus, args.impl)
    try:
        if args.impl == "reference":
            run_reference_arm(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
