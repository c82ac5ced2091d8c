"""The int8 tensor-core rate measurement (ie_cuda_mma_i8_peak): back-to-back
tcgen05.mma kind::i8 on every SM gives a rate near the B200's dense int8 peak
(4.5 POP/s nominal at the boost clock; the power cap may hold it lower), and
leaves no device error behind."""
import ctypes

import pytest

pytestmark = pytest.mark.gpu


def test_mma_i8_peak_plausible():
    from computeengine_b200 import _lib as L
    tops = ctypes.c_double()
    L.check(L.lib.ie_cuda_mma_i8_peak(40000, ctypes.byref(tops), None))
    assert 2500.0 < tops.value < 6000.0, tops.value
    assert L.take_device_error() == 0
