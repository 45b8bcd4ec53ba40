"""The C-ABI library loads on a CPU-only machine and exports every function include/fenix_b200.h
declares; status codes match the reference's fenix::Errc order (src/core/error.hpp:19-29)."""
import re

import pytest

import fenix_b200 as fx


def _declared(root):
    text = (root / "include" / "fenix_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)  # drop comments
    return sorted(set(re.findall(r"[\w*]\s+\**(fx_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(root):
    L = fx.lib()
    names = _declared(root)
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, f"not exported: {missing}"


def test_status_codes_follow_reference_errc(root):
    text = (root / "include" / "fenix_b200.h").read_text()
    order = ["FX_OK", "FX_INVALID_ARGUMENT", "FX_NOT_FOUND", "FX_IO_ERROR", "FX_FETCH_FAILED", "FX_DECODE_ERROR",
             "FX_UNSUPPORTED", "FX_UNIMPLEMENTED", "FX_INTERNAL"]
    for i, name in enumerate(order):
        assert re.search(rf"{name}\s*=\s*{i}\b", text), name


def test_create_rejects_missing_file_without_gpu_work(tmp_path):
    # On a CPU-only box the device check fails first; on a GPU box the file is missing. Either
    # way a clean status comes back through the ABI, never an exception or a crash.
    with pytest.raises(fx.FxError) as ei:
        fx.Net(str(tmp_path / "absent.fxweights"), patch=64)
    assert ei.value.code in (1, 3)


def test_tc_rate_rejects_bad_widths_before_device_work():
    # Argument checks come first: widths outside 16..256 or not a multiple of 16, a bad precision,
    # no runs or a null result pointer return FX_INVALID_ARGUMENT on any box, GPU or not.
    import ctypes as C

    b = C.c_double()
    for n in (0, 8, 24, 272):
        assert fx.lib().fx_tc_rate(0, fx.PREC_F16, n, 10.0, 1, C.byref(b), None) == fx.FX_INVALID_ARGUMENT
    assert fx.lib().fx_tc_rate(0, 7, 64, 10.0, 1, C.byref(b), None) == fx.FX_INVALID_ARGUMENT
    assert fx.lib().fx_tc_rate(0, fx.PREC_F16, 64, 10.0, 0, C.byref(b), None) == fx.FX_INVALID_ARGUMENT
    assert fx.lib().fx_tc_rate(0, fx.PREC_F16, 64, 10.0, 1, None, None) == fx.FX_INVALID_ARGUMENT
