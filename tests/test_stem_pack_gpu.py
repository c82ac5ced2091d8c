"""The stem re-layout kernel (space-to-depth 2x2 plus a 4-column unroll of an
NCHW uint8 image into 64-byte pixels) against a numpy statement of its
definition, bit-exact, for every supported channel count, both input sign
conventions (xor 0x80 turns int8 into biased uint8) and widths on both the
16-byte vector path and the byte path.  The whole stem convolution is checked
against the oracle's direct 7x7 conv in test_resnet_q8_gpu.py."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def stem_pack_numpy(x: np.ndarray, xor_mask: int) -> np.ndarray:
    """out[n][i][j][(ch*2+dy)*8 + 2b+dx] = x[n][ch][2i+dy][2(j+b-2)+dx] ^ mask,
    0 where j+b-2 is outside [0, w/2); channels 16c..63 are 0."""
    n, c, h, w = x.shape
    ho, wo = h // 2, w // 2
    xs = x ^ np.uint8(xor_mask)
    out = np.zeros((n, ho, wo, 64), np.uint8)
    for b in range(4):
        for dy in range(2):
            for dx in range(2):
                for ch in range(c):
                    chan = (ch * 2 + dy) * 8 + 2 * b + dx
                    src = xs[:, ch, dy::2, dx::2]  # [n, ho, wo], column jj
                    shift = b - 2                   # out column j reads jj = j + shift
                    j0, j1 = max(0, -shift), min(wo, wo - shift)
                    out[:, :, j0:j1, chan] = src[:, :, j0 + shift:j1 + shift]
    return out


CASES = [
    (2, 3, 224, 224, 0x00),   # ResNet stem, vector path
    (2, 3, 224, 224, 0x80),
    (1, 1, 6, 30, 0x00),      # w % 16 != 0: byte path
    (2, 2, 10, 64, 0x80),
    (1, 4, 8, 16, 0x00),
    (1, 3, 4, 520, 0x80),     # 260 output columns: more than one pixel per thread
    (3, 3, 2, 2, 0x00),       # one output pixel per row
]


@pytest.mark.parametrize("n,c,h,w,mask", CASES)
def test_stem_pack_matches_definition(n, c, h, w, mask):
    import torch
    from computeengine_b200 import _lib as L

    rng = np.random.default_rng(n * 1000 + c * 100 + w)
    x = rng.integers(0, 256, (n, c, h, w), dtype=np.uint8)
    xd = torch.from_numpy(x).cuda()
    out = torch.full((n, h // 2, w // 2, 64), 0xA5, dtype=torch.uint8, device="cuda")
    L.check(L.lib.ie_cuda_q8_stem_pack_input(xd.data_ptr(), out.data_ptr(), n, c, h, w, mask,
                                             None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), stem_pack_numpy(x, mask))
