"""The C++ ops (CudaConv2DOp, its depthwise form, CudaQLinearConv2DOp) driven
through the reference-shaped Op / OpRegistry interface on host tensors, checked
against the oracle: fp32 within max|err| <= 1e-3 * max|ref|, int8 bit-exact;
and the int8 post-training quantization flow (calibrate, quantize, int8 op,
dequantize) against the fp32 op; the pooling and Gemm ops through the registry
against the reference's own ops."""
import subprocess

import numpy as np
import pytest

from tests.backend_cpp import driver, read_dump

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def test_cpp_ops_match_oracle(oracle, tmp_path):
    r = subprocess.run([str(driver()), "gpu", str(tmp_path)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    t = read_dump(tmp_path)

    want = oracle.conv2d_f32(t["f32_x"], t["f32_w"], t["f32_b"], pads=(1, 1, 1, 1))
    err = float(np.abs(t["f32_y"] - want).max())
    assert err <= REL_TOL * float(np.abs(want).max()), err

    want = oracle.conv2d_f32(t["dw_x"], t["dw_w"], None, strides=(2, 2), group=32,
                             auto_pad="SAME_UPPER", depthwise=True)
    assert t["dw_y"].shape == want.shape
    err = float(np.abs(t["dw_y"] - want).max())
    assert err <= REL_TOL * float(np.abs(want).max()), err

    bias = t["q8_bias"].astype(np.int32)
    want = oracle.conv2d_q8(t["q8_x"], t["q8_w"], bias, t["q8_mult"], 128, 0, 0, 255,
                            pads=(1, 1, 1, 1))
    np.testing.assert_array_equal(t["q8_y"], want)
    assert (want == 0).any() and (want > 0).mean() > 0.2

    # int8 post-training quantization of a Conv2D + ReLU (calibrated on the
    # fp32 op): the int8 step is bit-exact with the oracle on the quantized
    # tensors and attributes the quantizer emitted, and the dequantized
    # output stays within the quantization error of the fp32 result
    # (max |err| <= 5% and mean |err| <= 0.5% of max |ref|: input, weight and
    # output steps of 1/255 of their ranges over a 288-term sum)
    zp_x, zp_y, qmin = (int(v) for v in t["ptq_zp"])
    assert zp_x not in (0, 128), "the calibrated input range should be asymmetric"
    want = oracle.conv2d_q8(t["ptq_xq"], t["ptq_wq"], t["ptq_bias"].astype(np.int32),
                            t["ptq_mult"], zp_x, zp_y, qmin, 255, pads=(1, 1, 1, 1))
    np.testing.assert_array_equal(t["ptq_yq"], want)
    ref = t["ptq_yf"]
    err = np.abs(t["ptq_ydq"] - ref)
    scale = float(np.abs(ref).max())
    assert err.max() <= 0.05 * scale, (err.max(), scale)
    assert err.mean() <= 0.005 * scale, (err.mean(), scale)


def test_cpp_q8_block_graph_device_resident(oracle, refconv, tmp_path):
    """A quantized ResNet bottleneck graph (int8 Conv2D nodes 1x1 -> 3x3 ->
    1x1, an int8 shortcut Add with ReLU and a 3x3 / 2 MaxPool2D) run by
    CudaExecutor with every int8 value in device memory, bit-exact with the
    oracle chain and the reference pool (the input's and conv1's zero points
    are neither 0 nor 128)."""
    r = subprocess.run([str(driver()), "gpu", str(tmp_path)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    t = read_dump(tmp_path)
    x = t["q8g_x"]
    p = [(t[f"q8g_qw{i}"], t[f"q8g_bias{i}"].astype(np.int32), t[f"q8g_mult{i}"]) for i in (1, 2, 3)]
    c1 = oracle.conv2d_q8(x, *p[0], 37, 10, 10, 255)
    c2 = oracle.conv2d_q8(c1, *p[1], 10, 0, 0, 255, pads=(1, 1, 1, 1))
    c3 = oracle.conv2d_q8(c2, *p[2], 0, 128, 0, 255)
    s = oracle.qadd(c3, 128, np.float32(0.5), x, 37, np.float32(0.75), 0, 0, 255)
    assert (s == 0).mean() < 0.9 and len(np.unique(s)) > 32
    # the graph ends in MaxPool2D 3x3 / 2, pads 1: the reference pool on the
    # same integers as floats
    rc, want = refconv.pool2d(s.astype(np.float32), (3, 3), (2, 2), (1, 1, 1, 1), kind="max")
    assert rc == 0
    np.testing.assert_array_equal(t["q8g_y"], want.astype(np.uint8))


def test_cpp_q8_network_to_logits(oracle, refconv, tmp_path):
    """A whole quantized network through CudaExecutor: int8 stem Conv2D 7x7 /
    2 (input zero point 128) -> int8 MaxPool -> bottleneck + int8 shortcut Add
    -> GlobalAvgPool of the int8 activation into fp32 -> Flatten -> Gemm.  The
    int8 part is recomputed with the oracle and the reference pool, the
    GlobalAvgPool by its rule (exact integer sum, double arithmetic, one fp32
    rounding), the Gemm by the reference GemmOp; logits within 1e-3 * max |ref|
    (the Gemm runs as bf16x3)."""
    r = subprocess.run([str(driver()), "gpu", str(tmp_path)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    t = read_dump(tmp_path)
    x = t["q8n_x"]
    p = [(t[f"q8n_nw{i}"], t[f"q8n_bias{i}"].astype(np.int32), t[f"q8n_mult{i}"]) for i in range(4)]
    s0 = oracle.conv2d_q8(x, *p[0], 128, 0, 0, 255, strides=(2, 2), pads=(3, 3, 3, 3))
    rc, pool = refconv.pool2d(s0.astype(np.float32), (3, 3), (2, 2), (1, 1, 1, 1), kind="max")
    assert rc == 0
    pool = pool.astype(np.uint8)
    c1 = oracle.conv2d_q8(pool, *p[1], 0, 0, 0, 255)
    c2 = oracle.conv2d_q8(c1, *p[2], 0, 0, 0, 255, pads=(1, 1, 1, 1))
    c3 = oracle.conv2d_q8(c2, *p[3], 0, 128, 0, 255)
    sm = oracle.qadd(c3, 128, np.float32(0.5), pool, 0, np.float32(0.75), 0, 0, 255)
    assert len(np.unique(sm)) > 16
    hw = sm.shape[2] * sm.shape[3]
    gap = (sm.astype(np.int64).sum(axis=(2, 3)).astype(np.float64) * np.float64(0.05)
           / np.float64(hw)).astype(np.float32)
    rc, want = refconv.gemm(gap, t["q8n_nfcw"], t["q8n_nfcb"], trans_b=1)
    assert rc == 0
    err = float(np.abs(t["q8n_y"] - want).max())
    assert err <= REL_TOL * float(np.abs(want).max()), err


def test_cpp_head_ops_match_reference(refconv, tmp_path):
    """MaxPool2D, AvgPool2D (ceil_mode, count_include_pad), GlobalAvgPool and
    Gemm (transB, bias) through the registry against the reference's own ops:
    pooling bit-exact, Gemm within 1e-3 * max |ref|."""
    r = subprocess.run([str(driver()), "gpu", str(tmp_path)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    t = read_dump(tmp_path)
    x = t["head_x"]
    rc, want = refconv.pool2d(x, (3, 3), (2, 2), (1, 1, 1, 1), kind="max")
    assert rc == 0
    np.testing.assert_array_equal(t["head_max"], want)
    rc, want = refconv.pool2d(x, (3, 3), (2, 2), (1, 1, 1, 1), ceil_mode=1, count_include_pad=1,
                              kind="avg")
    assert rc == 0
    np.testing.assert_array_equal(t["head_avg"], want)
    rc, want = refconv.pool2d(x, kind="global")
    assert rc == 0
    np.testing.assert_array_equal(t["head_gap"], want)
    rc, want = refconv.gemm(want.reshape(2, 16), t["head_wfc"], t["head_bfc"], trans_b=1)
    assert rc == 0
    err = float(np.abs(t["head_fc"] - want).max())
    assert err <= REL_TOL * float(np.abs(want).max()), err
    # int8 MaxPool2D, host NCHW I8: 2x3 kernel, strides (2, 1), pads
    # (0, 1, 1, 0), ceil_mode
    rc, want = refconv.pool2d(t["head_q8x"].astype(np.float32), (2, 3), (2, 1), (0, 1, 1, 0),
                              ceil_mode=1, kind="max")
    assert rc == 0
    np.testing.assert_array_equal(t["head_q8max"], want.astype(np.int8))


def test_conv_bn_relu_fusion_pass(oracle, tmp_path):
    """ConvBnReluFusionPass: the folded constants equal the reference's
    BatchNorm arithmetic applied to the weights (batch_norm_op.cpp:79-86,
    bit for bit), and the fused Conv2D + Relu run by CudaConv2DOp matches
    conv -> BatchNorm -> Relu (oracle conv, the reference's BatchNorm formula)
    within 1e-3 * max |ref|."""
    r = subprocess.run([str(driver()), "gpu", str(tmp_path)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    t = read_dump(tmp_path)
    f32 = np.float32
    inv = (1.0 / np.sqrt(t["bn_var"].astype(np.float64) + 1e-3)).astype(f32)
    gain = t["bn_scale"] * inv
    shift = t["bn_bias"] - t["bn_mean"] * gain
    np.testing.assert_array_equal(t["bn_wf"], t["bn_w"] * gain[:, None, None, None])
    np.testing.assert_array_equal(t["bn_bf"], t["bn_b"] * gain + shift)
    conv = oracle.conv2d_f32(t["bn_x"], t["bn_w"], t["bn_b"], pads=(1, 1, 1, 1))
    want = np.maximum(conv * gain[None, :, None, None] + shift[None, :, None, None], f32(0))
    err = float(np.abs(t["bn_y"] - want).max())
    assert err <= REL_TOL * float(np.abs(want).max()), err
    assert (want == 0).any() and (want > 0).mean() > 0.2


def test_conv_bn_add_relu_fusion(oracle, tmp_path):
    """The pass also fuses the bottleneck's shortcut Add: the fused Conv2D
    (folded BatchNorm, residual as fourth input, Relu) run by CudaConv2DOp
    matches conv -> BatchNorm -> Add -> Relu within 1e-3 * max |ref|."""
    r = subprocess.run([str(driver()), "gpu", str(tmp_path)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    t = read_dump(tmp_path)
    f32 = np.float32
    inv = (1.0 / np.sqrt(t["add_var"].astype(np.float64) + 1e-3)).astype(f32)
    gain = t["add_scale"] * inv
    shift = t["add_bias"] - t["add_mean"] * gain
    conv = oracle.conv2d_f32(t["add_x"], t["add_w"], t["add_b"], pads=(1, 1, 1, 1))
    bn = conv * gain[None, :, None, None] + shift[None, :, None, None]
    want = np.maximum(bn + t["add_r"], f32(0))
    err = float(np.abs(t["add_y"] - want).max())
    assert err <= REL_TOL * float(np.abs(want).max()), err


def test_cuda_executor_runs_fused_graph(oracle, tmp_path):
    """A ResNet-shaped graph (conv3x3+BN+Relu, max pool, conv1x1+BN, shortcut
    Add, Relu, global average pool, Flatten, Gemm) after the fusion pass, run
    by CudaExecutor with every intermediate value in device memory, against
    the same unfused network computed from the oracle convolution and numpy:
    max |err| <= 1e-3 * max |ref|; a second run reproduces the first."""
    from oracle.oracle import maxpool2d_nchw
    r = subprocess.run([str(driver()), "gpu", str(tmp_path)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    t = read_dump(tmp_path)
    f32 = np.float32

    def bn(v, p):
        inv = (1.0 / np.sqrt(t[p + "_var"].astype(np.float64) + 1e-5)).astype(f32)
        gain = t[p + "_scale"] * inv
        shift = t[p + "_bias"] - t[p + "_mean"] * gain
        return v * gain[None, :, None, None] + shift[None, :, None, None]

    c1 = oracle.conv2d_f32(t["net_x"], t["net_w1"], t["net_b1"], pads=(1, 1, 1, 1))
    r1 = np.maximum(bn(c1, "net_bn1"), f32(0))
    pool = maxpool2d_nchw(r1, 3, 2, 1).astype(f32)
    c2 = oracle.conv2d_f32(pool, t["net_w2"], None)
    r2 = np.maximum(bn(c2, "net_bn2") + pool, f32(0))
    gap = r2.mean(axis=(2, 3), dtype=np.float64).astype(f32)
    want = gap @ t["net_wfc"].T + t["net_bfc"]
    err = float(np.abs(t["net_y"] - want).max())
    assert err <= REL_TOL * float(np.abs(want).max()), err
