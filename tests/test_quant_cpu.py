"""The int8 post-training quantizer (C++ Int8QuantPlugin behind the reference's
QuantPlugin contract, src/core/plugin/quant_plugin.h:11-28) against a numpy
statement of its rules, bit for bit, on the driver's seeded tensors:

* weights: symmetric int8, one scale per output channel, scale = max|w| / 127
  (1 for an all-zero channel), q = clip(rne(w / scale), -127, 127);
* activations: asymmetric uint8 over [min(lo, 0), max(hi, 0)],
  scale = (hi - lo) / 255, zp = clip(rne(-lo / scale), 0, 255);
* min/max and 99.9th-percentile calibration over two batches (the percentile
  range drops an outlier);
* the CudaQLinearConv2DOp attributes: multiplier = fp32(s_x * s_w / s_y),
  bias = rne(b / (s_x * s_w)), ReLU6 folded into [zp_y, zp_y + rne(6 / s_y)];
* dequantize = (q - zp) * scale in fp32.
rne is round half to even; scale arithmetic in double, rounded to fp32."""
import subprocess

import numpy as np

from tests.backend_cpp import driver, read_dump

f32, f64 = np.float32, np.float64


def u8_params(lo, hi):
    lo, hi = min(f64(lo), 0.0), max(f64(hi), 0.0)
    scale = f32((hi - lo) / 255.0)
    if not scale > 0:
        scale = f32(1.0)
    zp = int(np.clip(np.rint(-lo / f64(scale)), 0, 255))
    return scale, zp


def test_quantizer_matches_numpy_rules(tmp_path):
    r = subprocess.run([str(driver()), "quant", str(tmp_path)], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    t = read_dump(tmp_path)

    # per-channel symmetric weights
    w = t["w"]
    amax = np.abs(w.reshape(16, -1)).max(axis=1)
    scales = (amax.astype(f64) / 127.0).astype(f32)
    scales[scales == 0] = 1.0
    np.testing.assert_array_equal(t["w_scales"], scales)
    wq = np.clip(np.rint(w.reshape(16, -1).astype(f64) / scales[:, None].astype(f64)), -127, 127)
    np.testing.assert_array_equal(t["wq"].reshape(16, -1), wq.astype(np.int8))
    assert (t["wq"][3] == 0).all() and t["wq"][5].reshape(-1)[7] == -127
    wdq = (t["wq"].reshape(16, -1).astype(f32) * scales[:, None]).reshape(w.shape)
    np.testing.assert_array_equal(t["wdq"], wdq)
    assert np.abs(t["wdq"] - w).max() <= scales.max() / 2 * (1 + 1e-6)

    # per-tensor symmetric
    st = f32(f64(np.abs(w).max()) / 127.0)
    assert t["wt_scale"][0] == st
    np.testing.assert_array_equal(t["wt"], np.clip(np.rint(w.astype(f64) / f64(st)), -127, 127)
                                  .astype(np.int8))

    # asymmetric activations
    x = t["x"]
    s_x, zp_x = u8_params(x.min(), x.max())
    assert t["x_params"][0] == s_x and int(t["x_params"][1]) == zp_x
    xq = np.clip(np.rint(x.astype(f64) / f64(s_x)) + zp_x, 0, 255).astype(np.uint8)
    np.testing.assert_array_equal(t["xq"], xq)
    np.testing.assert_array_equal(t["xdq"], (xq.astype(np.int32) - zp_x).astype(f32) * s_x)

    # calibration: min/max and the 99.9th percentile over both batches
    a = np.concatenate([t["a1"], t["a2"]])
    cal = t["cal"]
    assert cal[4] == a.min() and cal[5] == a.max()
    s_mm, zp_mm = u8_params(a.min(), a.max())
    assert cal[2] == s_mm and int(cal[3]) == zp_mm
    v = np.sort(a)
    k = lambda p: int(np.floor(p / 100.0 * (len(v) - 1) + 0.5))
    s_p, zp_p = u8_params(v[k(100.0 - 99.9)], v[k(99.9)])
    assert cal[0] == s_p and int(cal[1]) == zp_p
    assert s_p < s_mm / 5  # the 40.0 outlier is outside the percentile range

    # QLinearConv2D attributes (y range [0, 4], ReLU6)
    s_y, zp_y = u8_params(0.0, 4.0)
    mult = (f64(s_x) * scales.astype(f64) / f64(s_y)).astype(f32)
    np.testing.assert_array_equal(t["mult"], mult)
    bq = np.rint(t["bias"].astype(f64) / (f64(s_x) * scales.astype(f64)))
    np.testing.assert_array_equal(t["bias_q"], bq.astype(f32))
    qmin, qmax, zp_out = t["clamp"]
    assert int(qmin) == zp_y and int(zp_out) == zp_y
    assert int(qmax) == min(255, zp_y + int(np.rint(6.0 / f64(s_y))))
