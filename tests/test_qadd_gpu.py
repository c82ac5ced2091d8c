"""The int8 shortcut Add (ie_cuda_qadd) on the B200 against the oracle's
restatement: bit-exact, on the 16-byte vector path and the ragged element
path, uint8 / int8 operands and output, ties and saturation, on both the
64-bit arithmetic (multipliers' shifts at most 22 apart) and the 128-bit
one."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [
    # (count, ma, mb, zp_a, zp_b, zp_y, qmin, qmax, a_signed, b_signed, y_signed)
    (2 * 32 * 14 * 14, 0.5, 0.75, 128, 37, 0, 0, 255, False, False, False),
    (4096, 0.5, 0.25, 0, 0, 3, 3, 250, False, False, False),
    (1000, 0.37, 0.0213, 31, -5, 7, 0, 255, False, True, False),     # ragged length
    (4096, 1.5, 0.5, -3, 9, -4, -128, 127, True, True, True),
    (4096, 2.0 ** -40, 3.0, 0, 1, 0, 0, 255, False, False, False),
    # the 64-bit path's edge: shifts 22 apart, largest |x - zp| and significand
    (4096, 1.0, 2.0 ** -22, 255, 0, 0, 0, 255, False, False, False),
    (4096, 0.99999994, 0.99999994 * 2.0 ** -22, 0, 255, 128, 0, 255, False, False, False),
    (4096, 0.99999994, 0.99999994, -128, 127, 0, -128, 127, True, True, True),
    # 23 apart: the 128-bit path
    (4096, 1.0, 2.0 ** -23, 0, 0, 0, 0, 255, False, False, False),
]


@pytest.mark.parametrize("case", CASES, ids=range(len(CASES)))
def test_qadd_matches_oracle(oracle, case):
    import torch
    from computeengine_b200 import _lib as L
    count, ma, mb, zp_a, zp_b, zp_y, lo, hi, a_s, b_s, y_s = case
    rng = np.random.default_rng(count + zp_a)
    a = rng.integers(-128, 128, count).astype(np.int8) if a_s else rng.integers(0, 256, count).astype(np.uint8)
    b = rng.integers(-128, 128, count).astype(np.int8) if b_s else rng.integers(0, 256, count).astype(np.uint8)
    p = L.QAddParams()
    p.a_signed, p.zp_a, p.mult_a = int(a_s), zp_a, ma
    p.b_signed, p.zp_b, p.mult_b = int(b_s), zp_b, mb
    p.y_signed, p.zp_y, p.qmin, p.qmax = int(y_s), zp_y, lo, hi
    ad = torch.from_numpy(a.view(np.uint8)).cuda()
    bd = torch.from_numpy(b.view(np.uint8)).cuda()
    yd = torch.full((count,), 0x5A, dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_qadd(p, ad.data_ptr(), bd.data_ptr(), yd.data_ptr(), count,
                               torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    got = yd.cpu().numpy().view(np.int8 if y_s else np.uint8)
    want = oracle.qadd(a, zp_a, np.float32(ma), b, zp_b, np.float32(mb), zp_y, lo, hi, y_signed=y_s)
    np.testing.assert_array_equal(got, want)


def test_qadd_rejects_far_apart_multipliers():
    from computeengine_b200 import _lib as L
    p = L.QAddParams()
    p.mult_a, p.mult_b, p.qmin, p.qmax = 1.0, 2.0 ** -70, 0, 255
    rc = L.lib.ie_cuda_qadd(p, 16, 16, 16, 16, None)  # rejected before any device access
    assert rc == L.IE_UNSUPPORTED


LUT_CASES = [
    # (ma, mb, zp_a, zp_b, zp_y, qmin, qmax, a_signed, b_signed, y_signed)
    (1.0, 1.0, 128, 0, 0, 0, 255, False, False, False),          # the ResNet shortcut Add
    (0.5, 0.75, 128, 37, 3, 3, 250, False, False, False),
    (1.5, 0.5, -3, 9, -4, -128, 127, True, True, True),
    (2.0 ** -40, 3.0, 0, 1, 0, 0, 255, False, False, False),     # 128-bit arithmetic
]


@pytest.mark.parametrize("case", LUT_CASES, ids=range(len(LUT_CASES)))
def test_qadd_table_path_matches_oracle(oracle, case):
    """Tensors of at least 4M bytes take the table kernel (qadd_lut_u8): every
    one of the 65536 byte pairs appears 64 times, shuffled, plus a few more
    elements; bit-exact with the oracle."""
    import torch
    from computeengine_b200 import _lib as L
    ma, mb, zp_a, zp_b, zp_y, lo, hi, a_s, b_s, y_s = case
    rng = np.random.default_rng(65536 + zp_a)
    pairs = np.concatenate([np.tile(np.arange(65536), 64), rng.integers(0, 65536, 48 * 16)])
    pairs = rng.permutation(pairs)
    count = pairs.size
    assert count % 16 == 0 and count >= 1 << 22
    a = (pairs >> 8).astype(np.uint8)
    b = (pairs & 255).astype(np.uint8)
    a_v = a.view(np.int8) if a_s else a
    b_v = b.view(np.int8) if b_s else b
    p = L.QAddParams()
    p.a_signed, p.zp_a, p.mult_a = int(a_s), zp_a, ma
    p.b_signed, p.zp_b, p.mult_b = int(b_s), zp_b, mb
    p.y_signed, p.zp_y, p.qmin, p.qmax = int(y_s), zp_y, lo, hi
    ad = torch.from_numpy(a).cuda()
    bd = torch.from_numpy(b).cuda()
    yd = torch.full((count,), 0x5A, dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_qadd(p, ad.data_ptr(), bd.data_ptr(), yd.data_ptr(), count,
                               torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    got = yd.cpu().numpy().view(np.int8 if y_s else np.uint8)
    want = oracle.qadd(a_v, zp_a, np.float32(ma), b_v, zp_b, np.float32(mb), zp_y, lo, hi, y_signed=y_s)
    np.testing.assert_array_equal(got, want)
