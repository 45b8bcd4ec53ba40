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


def test_tc_rate_narrow_mmas(cuda_torch):
    """The MMA shapes of the narrow conv layers: N = 32 .. 256 columns. Every width runs within the
    dense nominal, and the 32-column shape is clearly slower than the widest: its A tile's
    shared-memory read is spread over a quarter of the columns of math of N = 128."""
    rates = {n: fx.tc_rate("f16", n, 20.0, 3)[0] for n in (32, 64, 96, 128, 192, 256)}
    print("f16 tcgen05 rate by N:", {n: round(r) for n, r in rates.items()})
    top = max(rates.values())
    assert all(r > 50.0 for r in rates.values())
    assert top < 2400.0
    assert rates[32] < 0.8 * top


def test_tc_rate_arguments(cuda_torch):
    import ctypes as C

    b = C.c_double()
    for n in (0, 8, 24, 272):
        assert fx.lib().fx_tc_rate(0, 2, n, 10.0, 1, C.byref(b), None) == fx.FX_INVALID_ARGUMENT
