"""Edge cases of the whole path against the oracle (f16 operands, the reference's GPU precision):
volumes smaller than one tile, ragged extents, a one-class sigmoid head, the other softmax
channel, a single conv per stage, and the argument checks of the C ABI. Tiles are 64^3 (the
reference accepts patches that are multiples of 64)."""
import ctypes as C

import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import make_plain_unet
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

FEATS = (16, 32, 64, 128)
TOL = 1e-2


def run(tmp_path, shape, P, ov=0.5, ncls=2, nconv=2, channel=1, sigmoid=0, seed=4, batch=2):
    w = make_plain_unet(tmp_path / "e.fxweights", FEATS, nconv=nconv, ncls=ncls, seed=seed)
    vol = fx.synth_spiral(shape, seed + 100, fx.SPIRAL_CONFIG1)
    net = fx.Net(w, P, max_batch=batch, precision="f16")
    prob, u8 = net.predict_volume(vol, overlap=ov, batch=batch, channel=channel, sigmoid=sigmoid)
    net.close()
    want = orc.Net(w).predict_surface(vol, P, ov, channel=channel, sigmoid=sigmoid)
    err = float(np.abs(prob - want).max())
    du8 = int(np.abs(u8.astype(int) - orc.prob_to_u8(want).astype(int)).max())
    return err, du8, prob


def test_volume_smaller_than_tile(cuda_torch, tmp_path):
    err, du8, _ = run(tmp_path, (20, 24, 28), 64)  # one tile, edge-clamped reads on every axis
    assert err <= TOL and du8 <= 4


def test_ragged_extents(cuda_torch, tmp_path):
    err, du8, _ = run(tmp_path, (150, 70, 181), 64, ov=0.25)  # last starts clamped to dim - P
    assert err <= TOL and du8 <= 4


def test_sigmoid_one_class_head(cuda_torch, tmp_path):
    err, du8, prob = run(tmp_path, (96, 72, 80), 64, ncls=1, sigmoid=1)
    assert err <= TOL and du8 <= 4
    assert prob.min() >= 0.0 and prob.max() <= 1.0


def test_softmax_channel_zero(cuda_torch, tmp_path):
    err, du8, _ = run(tmp_path, (80, 96, 72), 64, channel=0)
    assert err <= TOL and du8 <= 4


def test_one_conv_per_stage(cuda_torch, tmp_path):
    err, du8, _ = run(tmp_path, (80, 72, 88), 64, nconv=1)
    assert err <= TOL and du8 <= 4


def test_abi_argument_checks(cuda_torch, tmp_path):
    L = fx.lib()
    w = make_plain_unet(tmp_path / "e.fxweights", FEATS, seed=1)
    net = fx.Net(w, 64, max_batch=2, precision="f16")
    vol = np.zeros((8, 8, 8), np.uint8)
    vp = vol.ctypes.data_as(C.POINTER(C.c_uint8))
    out = np.zeros(vol.shape, np.uint8)
    op = out.ctypes.data_as(C.POINTER(C.c_uint8))
    ok = fx.InferOpts(64, 0.5, 1, 0, 2, 0)
    assert L.fx_predict_volume(net.handle, vp, 0, 8, 8, C.byref(ok), None, op) == 1  # empty volume
    assert L.fx_predict_volume(net.handle, None, 8, 8, 8, C.byref(ok), None, op) == 1  # null input
    wrong = fx.InferOpts(128, 0.5, 1, 0, 2, 0)  # patch differs from the net's
    assert L.fx_predict_volume(net.handle, vp, 8, 8, 8, C.byref(wrong), None, op) == 1
    odd = fx.InferOpts(96, 0.5, 1, 0, 2, 0)  # not a multiple of 64 (the reference's check)
    assert L.fx_predict_volume(net.handle, vp, 8, 8, 8, C.byref(odd), None, op) == 1
    assert L.fx_last_error()  # every failure leaves a message
    net.close()
