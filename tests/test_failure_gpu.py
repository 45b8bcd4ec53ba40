"""Failure detection on the device without a GPU fault: every barrier wait of the conv kernel is
bounded, and a wait that runs out sets a status word, ends the launch and leaves the context
usable. fx_selftest_wait_timeout runs one conv launch whose MMA warp waits on a barrier nothing
arrives at, with a short limit; the host reads the status back, then the same process runs a
normal forward. (The reference's counterpart is its worker error path, src/ml/infer.hpp:675-808,
where a failed step surfaces as an Expected error instead of a hang.)"""
import ctypes as C
import time

import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import make_plain_unet
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

# the first bounded wait to give up records its code (ptx.cuh): the MMA warp's stage wait (0x100) or
# the epilogue's accumulator wait (0x300), which starts at the same moment
TIMEOUT_CODES = (0x100, 0x300)


def test_bounded_wait_times_out_and_context_survives(cuda_torch, tmp_path):
    st = C.c_uint32(0)
    t0 = time.perf_counter()
    fx.check(fx.lib().fx_selftest_wait_timeout(0, 50_000_000, C.byref(st)))  # 50 ms limit
    dt = time.perf_counter() - t0
    assert st.value in TIMEOUT_CODES, hex(st.value)
    assert dt < 10.0
    # the context is intact: a whole forward still runs and matches the oracle
    w = make_plain_unet(tmp_path / "f.fxweights", (16, 32, 64, 128), seed=2)
    vol = fx.synth_spiral((64, 64, 64), 5, fx.SPIRAL_CONFIG1)
    net = fx.Net(w, 64, max_batch=1, precision="f16")
    prob, _ = net.predict_volume(vol, overlap=0.5, batch=1)
    fx.check(fx.lib().fx_net_device_status(net.handle))
    net.close()
    want = orc.Net(w).predict_surface(vol, 64, 0.5)
    assert float(np.abs(prob - want).max()) <= 1e-2


def test_selftest_argument_checks(cuda_torch):
    st = C.c_uint32(0)
    assert fx.lib().fx_selftest_wait_timeout(0, 0, C.byref(st)) == fx.FX_INVALID_ARGUMENT
    assert fx.lib().fx_selftest_wait_timeout(999, 1000, C.byref(st)) == fx.FX_INVALID_ARGUMENT
