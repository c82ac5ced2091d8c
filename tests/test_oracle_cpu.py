"""The CPU oracle, pinned before it is trusted:
* fp32: against the reference's own golden vectors (PyTorch float32,
  tests/data/traditional_reference.h in the reference) and against the
  reference's Conv2DOp compiled from its sources, on the geometry the
  reference tests (pads, SAME_UPPER / SAME_LOWER, dilation, groups);
* int8 accumulation: against the reference Conv2DOp on integer-valued data
  (exact in fp32 while partial sums stay below 2^24);
* int8 requantize: against an independent float64 restatement, on ties and
  saturation edges (the reference has no int8 conv, so this rule is pinned
  only by its own definition)."""
import numpy as np
import pytest


def test_golden_conv_and_depthwise(oracle, golden):
    y = oracle.conv2d_f32(golden["kConvInput"], golden["kConvWeight"], golden["kConvBias"],
                          pads=(1, 1, 1, 1))
    np.testing.assert_allclose(y, golden["kConvExpected"], atol=1e-5, rtol=0)
    y = oracle.conv2d_f32(golden["kConvInput"], golden["kConvWeight"], None, pads=(1, 1, 1, 1))
    np.testing.assert_allclose(y, golden["kConvExpected"] - golden["kConvBias"].reshape(1, 3, 1, 1),
                               atol=1e-5, rtol=0)
    y = oracle.conv2d_f32(golden["kConvInput"], golden["kConvWeight"], golden["kConvBias"],
                          auto_pad="SAME_UPPER")
    np.testing.assert_allclose(y, golden["kConvExpected"], atol=1e-5, rtol=0)
    y = oracle.conv2d_f32(golden["kDepthwiseInput"], golden["kDepthwiseWeight"],
                          golden["kDepthwiseBias"], group=2, depthwise=True)
    np.testing.assert_allclose(y, golden["kDepthwiseExpected"], atol=1e-5, rtol=0)


def test_reference_known_answers(oracle):
    # grouped manual values (traditional_ops_test.cpp GroupedMatchesManualValues)
    x = np.arange(1, 9, dtype=np.float32).reshape(1, 2, 2, 2)
    w = np.array([2, 3], np.float32).reshape(2, 1, 1, 1)
    y = oracle.conv2d_f32(x, w, None, group=2)
    np.testing.assert_array_equal(y.ravel(), [2, 4, 6, 8, 15, 18, 21, 24])
    # SAME_UPPER / SAME_LOWER direction and dilation (Conv2DAutoPadDirectionAndDilation)
    x = np.arange(1, 17, dtype=np.float32).reshape(1, 1, 4, 4)
    ones = np.ones((1, 1, 3, 3), np.float32)
    up = oracle.conv2d_f32(x, ones, None, strides=(2, 2), auto_pad="SAME_UPPER")
    lo = oracle.conv2d_f32(x, ones, None, strides=(2, 2), auto_pad="SAME_LOWER")
    assert up.shape == lo.shape == (1, 1, 2, 2)
    assert up.ravel()[0] == 1 + 2 + 3 + 5 + 6 + 7 + 9 + 10 + 11
    assert lo.ravel()[3] == 6 + 7 + 8 + 10 + 11 + 12 + 14 + 15 + 16
    x3 = np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3)
    y = oracle.conv2d_f32(x3, np.ones((1, 1, 2, 2), np.float32), None, dilations=(2, 2))
    assert y.shape == (1, 1, 1, 1) and y.ravel()[0] == 1 + 3 + 7 + 9


def test_error_codes_match_reference(oracle):
    from oracle.oracle import INVALID_ARGUMENT, OracleError
    with pytest.raises(OracleError) as e:
        oracle.resolve((1, 2, 5, 5), (3, 2, 3, 3), group=4)
    assert e.value.code == INVALID_ARGUMENT
    with pytest.raises(OracleError) as e:
        oracle.resolve((1, 2, 3, 3), (2, 1, 2, 2), group=1, depthwise=True)
    assert e.value.code == INVALID_ARGUMENT


GEOMETRIES = [
    dict(x=(2, 3, 9, 11), w=(4, 3, 3, 3), pads=(1, 1, 1, 1)),
    dict(x=(1, 4, 8, 8), w=(6, 2, 3, 3), group=2, strides=(2, 2), pads=(0, 1, 1, 0)),
    dict(x=(1, 2, 7, 7), w=(2, 1, 3, 3), group=2, dilations=(2, 2), auto_pad="SAME_LOWER"),
    dict(x=(1, 3, 10, 6), w=(5, 3, 2, 4), strides=(3, 1), auto_pad="SAME_UPPER"),
    dict(x=(2, 8, 6, 6), w=(8, 1, 3, 3), group=8, pads=(1, 1, 1, 1), depthwise=True),
]


@pytest.mark.parametrize("g", GEOMETRIES, ids=range(len(GEOMETRIES)))
def test_fp32_matches_reference_conv(oracle, refconv, g):
    rng = np.random.default_rng(3)
    x = rng.normal(size=g["x"]).astype(np.float32)
    w = rng.normal(size=g["w"]).astype(np.float32)
    b = rng.normal(size=g["w"][0]).astype(np.float32)
    kw = {k: v for k, v in g.items() if k not in ("x", "w")}
    rc, want = refconv.conv2d(x, w, b, **kw)
    assert rc == 0
    got = oracle.conv2d_f32(x, w, b, **kw)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("g", GEOMETRIES, ids=range(len(GEOMETRIES)))
def test_reference_wrapper_dims_and_threads(refconv, g):
    """The wrapper's output dims for explicit padding (the reference's own
    formula) equal the library's shape query, and a threaded batch call
    (one image per thread) equals the images run one by one."""
    from oracle.oracle import RefConv
    rng = np.random.default_rng(5)
    xs = (3,) + tuple(g["x"][1:])
    x = rng.normal(size=xs).astype(np.float32)
    w = rng.normal(size=g["w"]).astype(np.float32)
    kw = {k: v for k, v in g.items() if k not in ("x", "w")}
    full = dict(strides=(1, 1), dilations=(1, 1), pads=(0, 0, 0, 0), auto_pad="NOTSET")
    full.update({k: v for k, v in kw.items() if k in full})
    known = RefConv._explicit_dims(x.shape, w.shape, full["strides"], full["dilations"],
                                   full["pads"], full["auto_pad"])
    rc, whole = refconv.conv2d(x, w, None, nthreads=3, **kw)
    assert rc == 0
    if known is not None:
        assert tuple(whole.shape) == tuple(known)
    parts = []
    for i in range(x.shape[0]):
        rc, y = refconv.conv2d(x[i:i + 1], w, None, **kw)
        assert rc == 0
        parts.append(y)
    np.testing.assert_array_equal(whole, np.concatenate(parts))


def test_reference_wrapper_keeps_error_codes(refconv):
    """Shapes the formula cannot vouch for go to the library, which answers
    with the reference's own error code."""
    from oracle.oracle import INVALID_ARGUMENT
    x = np.zeros((2, 3, 4, 4), np.float32)
    rc, y = refconv.conv2d(x, np.zeros((4, 3, 7, 7), np.float32))  # kernel > padded input
    assert rc == INVALID_ARGUMENT and y is None
    rc, y = refconv.conv2d(x, np.zeros((4, 5, 3, 3), np.float32))  # channel mismatch
    assert rc == INVALID_ARGUMENT and y is None


@pytest.mark.parametrize("g", GEOMETRIES[:4], ids=range(4))
def test_int8_accumulators_match_reference_conv(oracle, refconv, g):
    """Integer-valued fp32 through the reference conv is exact below 2^24, so
    it pins the int8 oracle's accumulation (geometry, padding = real zero)."""
    rng = np.random.default_rng(4)
    zp = 128
    x = rng.integers(0, 256, g["x"]).astype(np.uint8)
    w = rng.integers(-127, 128, g["w"]).astype(np.int8)
    kw = {k: v for k, v in g.items() if k not in ("x", "w")}
    rc, want = refconv.conv2d(x.astype(np.float32) - zp, w.astype(np.float32), None, **kw)
    assert rc == 0
    _, acc = oracle.conv2d_q8(x, w, None, np.ones(g["w"][0], np.float32), zp, 0, 0, 255,
                              want_acc=True, **kw)
    np.testing.assert_array_equal(acc, want.astype(np.int64))


def _requant_exact(acc, bias, mult, zp, qmin, qmax):
    """Independent restatement with Python fractions: round half away from zero
    of the exact product (int32 acc + bias) * (exact value of the fp32 mult)."""
    from fractions import Fraction
    t = int(np.int32(np.int64(acc) + np.int64(bias)))
    v = Fraction(t) * Fraction(float(np.float32(mult)))
    a = abs(v)
    r = int(a + Fraction(1, 2)) if v >= 0 else -int(a + Fraction(1, 2))
    return int(min(max(r + zp, qmin), qmax))


def test_requantize_edges(oracle):
    rng = np.random.default_rng(9)
    cases = []
    for m in (0.5, 0.25, 1.5, 3 * 2.0 ** -9, 0.0037, 1e-4, 7.0):
        for acc in list(range(-20, 21)) + [2 ** 24 + 1, -(2 ** 24) - 3, 2 ** 30, -(2 ** 31) + 5]:
            cases.append((acc, 0, m))
    for _ in range(5000):
        cases.append((int(rng.integers(-2 ** 26, 2 ** 26)), int(rng.integers(-5000, 5000)),
                      float(np.float32(rng.uniform(1e-5, 0.05)))))
    # products a hair below / at / above a tie
    cases.append((1, 0, float(np.float32(0.5) - np.float32(2.0 ** -25))))
    cases.append((-1, 0, float(np.float32(0.5) - np.float32(2.0 ** -25))))
    cases.append((3, 0, float(np.float32(0.5))))
    cases.append((-3, 0, float(np.float32(0.5))))
    cases.append((2 ** 24 + 1, 0, float(np.float32(0.5))))
    for m in (0.75, 1.0, 3.0, 2.0 ** 20, 2.0 ** 31, 2.0 ** 40, 2.0 ** -40, 2.0 ** -62):
        for acc in (-7, -1, 0, 1, 5, 2 ** 31 - 1, -(2 ** 31)):
            cases.append((acc, 0, m))
    for zp, lo, hi in ((0, 0, 255), (3, 3, 123), (-7, -128, 127), (100, 0, 255)):
        for acc, b, m in cases:
            assert oracle.requantize(acc, b, m, zp, lo, hi) == _requant_exact(acc, b, m, zp, lo, hi), \
                (acc, b, m, zp, lo, hi)


def test_qadd_matches_fraction_restatement(oracle):
    """The int8 Add rule (round half away from zero of the exact sum of the two
    rescaled operands, then zero point and clamp), checked on random values and
    on multipliers that make exact .5 ties of either sign."""
    import math
    from fractions import Fraction as F
    rng = np.random.default_rng(7)

    def rha(v):
        return int(math.floor(abs(v) + F(1, 2))) * (1 if v >= 0 else -1)

    for (ma, mb, zp_a, zp_b, zp_y, lo, hi, a_s, b_s, y_s) in [
            (0.37, 0.0213, 31, -5, 7, 0, 255, False, True, False),
            (0.5, 0.25, 128, 0, 0, 0, 255, False, False, False),      # ties
            (0.5, 1.5, -3, 9, -4, -128, 127, True, True, True),      # ties, signed output
            (2.0 ** -40, 3.0, 0, 1, 0, 0, 255, False, False, False),  # shifts 42 apart
            (0.0, 0.8, 5, 6, 1, 0, 200, False, False, False)]:        # a vanishing term
        a = rng.integers(-128, 128, 700).astype(np.int8) if a_s else rng.integers(0, 256, 700).astype(np.uint8)
        b = rng.integers(-128, 128, 700).astype(np.int8) if b_s else rng.integers(0, 256, 700).astype(np.uint8)
        y = oracle.qadd(a, zp_a, np.float32(ma), b, zp_b, np.float32(mb), zp_y, lo, hi, y_signed=y_s)
        want = [min(max(rha((int(av) - zp_a) * F(float(np.float32(ma))) +
                            (int(bv) - zp_b) * F(float(np.float32(mb)))) + zp_y, lo), hi)
                for av, bv in zip(a, b)]
        np.testing.assert_array_equal(y.astype(np.int64), np.array(want, np.int64))
