"""The C ABI library loads on a machine without a GPU, exports every function
include/ie_cuda_conv.h declares, and its host-only geometry (ie_conv2d_resolve)
agrees with the oracle's restatement of conv2d_forward's checks."""
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def header_functions():
    text = (ROOT / "include" / "ie_cuda_conv.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ie_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    import ctypes
    from computeengine_b200 import _lib
    names = header_functions()
    assert len(names) >= 20
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def _desc(**kw):
    from computeengine_b200 import _lib as L
    from tests.qconv import desc_for
    base = dict(n=1, c=2, h=5, w=5, m=3, kh=3, kw=3)
    base.update({k: kw[k] for k in list(kw) if k in base})
    return desc_for(L, base["n"], base["c"], base["h"], base["w"], base["m"], base["kh"], base["kw"],
                    kw.get("stride", (1, 1)), kw.get("pads", (0, 0, 0, 0)), kw.get("dil", (1, 1)),
                    kw.get("group", 1), kw.get("auto_pad", 0), kw.get("depthwise", 0))


GEOMS = [
    dict(),
    dict(pads=(1, 1, 1, 1)),
    dict(h=4, w=4, c=1, m=1, stride=(2, 2), auto_pad=2),
    dict(h=4, w=4, c=1, m=1, stride=(2, 2), auto_pad=3),
    dict(h=3, w=3, c=1, m=1, kh=2, kw=2, dil=(2, 2)),
    dict(h=7, w=9, c=4, m=8, kh=3, kw=1, stride=(2, 3), pads=(0, 2, 1, 0)),
    dict(c=4, m=6, group=2),
    dict(auto_pad=1, h=9, w=9),
    dict(h=2, w=2),                    # kernel exceeds input
    dict(group=4),                     # group does not divide c
    dict(c=4, m=4, group=2, depthwise=1),  # depthwise needs group == c
]


@pytest.mark.parametrize("g", GEOMS, ids=range(len(GEOMS)))
def test_resolve_matches_oracle(oracle, g):
    from computeengine_b200 import _lib as L
    from oracle.oracle import OracleError
    d = _desc(**g)
    s = L.ConvShape()
    rc = L.lib.ie_conv2d_resolve(d, -1, s)
    inv = {0: "NOTSET", 1: "VALID", 2: "SAME_UPPER", 3: "SAME_LOWER"}
    try:
        geo = oracle.resolve((d.n, d.c, d.h, d.w), (d.m, d.c // max(d.group, 1), d.kh, d.kw),
                             strides=(d.stride_h, d.stride_w), dilations=(d.dil_h, d.dil_w),
                             pads=(d.pad_top, d.pad_left, d.pad_bottom, d.pad_right),
                             group=d.group, auto_pad=inv[d.auto_pad], depthwise=bool(d.depthwise))
        want = 0
    except OracleError as e:
        want = e.code
    assert rc == want
    if rc == 0:
        assert (s.out_h, s.out_w) == (geo.out_h, geo.out_w)
        assert (s.pad_top, s.pad_left, s.pad_bottom, s.pad_right) == \
            (geo.pad_t, geo.pad_l, geo.pad_b, geo.pad_r)


def test_bias_length_and_error_text():
    from computeengine_b200 import _lib as L
    d = _desc()
    s = L.ConvShape()
    assert L.lib.ie_conv2d_resolve(d, 2, s) == L.IE_INVALID_ARGUMENT
    assert b"bias" in L.lib.ie_cuda_last_error()
    assert L.lib.ie_conv2d_resolve(d, 3, s) == L.IE_OK


def test_packed_sizes():
    from computeengine_b200 import _lib as L
    # packed weights, then the int32 per-channel weight sums (m rounded up to 16)
    d = _desc(c=64, m=128, h=28, w=28, pads=(1, 1, 1, 1))
    assert L.lib.ie_cuda_q8_packed_weight_bytes(d) == 128 * 9 * 64 + 4 * 128
    assert L.lib.ie_cuda_q8_halo_input_bytes(d) == 1 * 30 * 30 * 64
    d = _desc(c=3, m=64, kh=7, kw=7)
    assert L.lib.ie_cuda_q8_packed_weight_bytes(d) == 64 * 49 * 32 + 4 * 64
    assert L.lib.ie_cuda_f32_packed_weight_bytes(d) == 64 * 49 * 2 * 16 * 2
    d = _desc(c=24, m=40, h=9, w=7, kh=3, kw=3, stride=(2, 2), pads=(1, 0, 2, 1))
    assert L.lib.ie_cuda_q8_packed_weight_bytes(d) == 40 * 9 * 32 + 4 * 48
    assert L.lib.ie_cuda_q8_halo_input_bytes(d) == 12 * 8 * 32
    sd = L.ConvDesc()
    assert L.lib.ie_cuda_q8_stem_desc(8, 3, 224, 224, 64, sd) == 0
    assert (sd.c, sd.h, sd.kh, sd.kw, sd.pad_top, sd.pad_bottom) == (64, 112, 4, 1, 2, 1)
    assert L.lib.ie_cuda_q8_stem_desc(8, 5, 224, 224, 64, sd) == L.IE_UNSUPPORTED


def test_tile_policy_values():
    """ie_cuda_set_tile_policy is host-only: returns the previous policy and
    rejects unknown values."""
    from computeengine_b200 import _lib as L
    prev = L.set_tile_policy(L.IE_TILE_DEFAULT)
    try:
        assert L.set_tile_policy(L.IE_TILE_DEFAULT) == L.IE_TILE_DEFAULT
        with pytest.raises(L.CudaConvError):
            L.set_tile_policy(7)
        assert L.set_tile_policy(L.IE_TILE_FILL) == L.IE_TILE_DEFAULT
    finally:
        L.set_tile_policy(prev)


def test_mma_peak_rejects_bad_arguments():
    """ie_cuda_mma_i8_peak checks its arguments before any CUDA call."""
    import ctypes
    from computeengine_b200 import _lib as L
    out = ctypes.c_double()
    assert L.lib.ie_cuda_mma_i8_peak(5, ctypes.byref(out), None) == L.IE_INVALID_ARGUMENT
    assert L.lib.ie_cuda_mma_i8_peak(40000, None, None) == L.IE_INVALID_ARGUMENT
