"""The measured tcgen05 rate (fx_tc_peak, the tensor roofline's denominator): e4m3 runs at about
twice the 16-bit rate, both within the B200's dense nominal (4.5 / 2.25 PFLOP/s) and well above
what a fraction of the SMs could deliver."""
import pytest

import fenix_b200 as fx

pytestmark = pytest.mark.gpu


def test_tc_peak_rates(cuda_torch):
    f8, f8m = fx.tc_peak("fp8", 20.0, 3)
    f16, _ = fx.tc_peak("f16", 20.0, 3)
    bf16, _ = fx.tc_peak("bf16", 20.0, 3)
    print(f"tcgen05 dense: e4m3 {f8:.0f} TFLOP/s (mean {f8m:.0f}), f16 {f16:.0f}, bf16 {bf16:.0f}")
    assert 1000.0 < f8 < 4600.0
    assert 500.0 < f16 < 2300.0 and 500.0 < bf16 < 2300.0
    assert 1.7 < f8 / f16 < 2.3
    assert f8m <= f8 + 1e-6


def test_tc_peak_arguments(cuda_torch):
    import ctypes as C

    b = C.c_double()
    assert fx.lib().fx_tc_peak(0, 7, 10.0, 1, C.byref(b), None) == fx.FX_INVALID_ARGUMENT
    assert fx.lib().fx_tc_peak(0, 1, 0.0, 1, C.byref(b), None) == fx.FX_INVALID_ARGUMENT
