"""Pooling geometry of the head ops without a GPU: ie_pool2d_resolve (the
C ABI's restatement of resolve_pool_geometry, pool_ops.cpp:24-61) gives the
same output extent as the reference MaxPool2DOp compiled from its sources,
and rejects the same shapes, over seeded random geometries with every
auto_pad mode and ceil_mode."""
import numpy as np
import pytest

AUTO = {"NOTSET": 0, "VALID": 1, "SAME_UPPER": 2, "SAME_LOWER": 3}


def test_pool_resolve_matches_reference(refconv):
    from computeengine_b200 import _lib as L
    rng = np.random.default_rng(0)
    checked = rejected = 0
    for _ in range(300):
        h, w = (int(v) for v in rng.integers(1, 12, 2))
        kh, kw = (int(v) for v in rng.integers(1, 6, 2))
        sh, sw = (int(v) for v in rng.integers(1, 4, 2))
        pads = [int(v) for v in rng.integers(0, 3, 4)]
        auto = list(AUTO)[int(rng.integers(0, 4))]
        ceil_mode = int(rng.integers(0, 2))
        d = L.PoolDesc()
        d.n, d.c, d.h, d.w, d.kh, d.kw, d.stride_h, d.stride_w = 1, 1, h, w, kh, kw, sh, sw
        d.pad_top, d.pad_left, d.pad_bottom, d.pad_right = pads
        d.auto_pad, d.ceil_mode = AUTO[auto], ceil_mode
        s = L.ConvShape()
        rc = L.lib.ie_pool2d_resolve(d, s)
        x = np.zeros((1, 1, h, w), np.float32)
        rrc, y = refconv.pool2d(x, (kh, kw), (sh, sw), pads, auto, ceil_mode)
        assert rc == rrc, (h, w, kh, kw, sh, sw, pads, auto, ceil_mode)
        if rc == 0:
            assert (s.out_h, s.out_w) == y.shape[2:]
            checked += 1
        else:
            rejected += 1
    assert checked > 150 and rejected > 5
