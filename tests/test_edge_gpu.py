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


@pytest.mark.parametrize("bias1,channel,sigmoid,want", [
    (np.inf, 1, 0, 0.0),    # softmax over [finite, +inf] = [0, nan] -> nan_to_num -> 0
    (np.inf, 0, 0, 0.0),    # the other channel: 0 / nan -> 0
    (-np.inf, 1, 0, 0.0),   # exp(-inf) = 0
    (-np.inf, 0, 0, 1.0),
    (np.nan, 1, 0, 0.0),    # NaN logits everywhere -> 0
    (np.inf, 0, 1, 1.0),    # sigmoid(+inf) = 1
    (np.nan, 0, 1, 0.0),
])
def test_head_scrubs_nan_and_inf(cuda_torch, tmp_path, bias1, channel, sigmoid, want):
    """A non-finite head bias makes every logit of that class non-finite; the fused head kernel
    scrubs the probability as the reference's nan_to_num(nan=0, posinf=1, neginf=0) does
    (src/ml/infer.hpp:760-767), and the oracle gives the same bytes."""
    from fenix_b200.weights import plain_unet_params, write_fxweights

    ncls = 1 if sigmoid else 2
    prm = plain_unet_params(FEATS, ncls=ncls, seed=7)
    key = f"decoder.seg_layers.{len(FEATS) - 2}.bias"
    prm[key] = prm[key].copy()
    prm[key][-1 if not sigmoid else 0] = bias1
    w = tmp_path / "nan.fxweights"
    write_fxweights(w, prm)
    vol = fx.synth_spiral((72, 64, 80), 11, fx.SPIRAL_CONFIG1)
    net = fx.Net(w, 64, max_batch=2, precision="f16")
    prob, u8 = net.predict_volume(vol, overlap=0.5, batch=2, channel=channel, sigmoid=sigmoid)
    net.close()
    assert np.isfinite(prob).all()
    # a constant tile probability survives the blend up to the rounding of the weight sums
    assert float(np.abs(prob - np.float32(want)).max()) <= 1e-6, (prob.min(), prob.max())
    oracle = orc.Net(w).predict_surface(vol, 64, 0.5, channel=channel, sigmoid=sigmoid)
    assert float(np.abs(prob - oracle).max()) <= 1e-6
    assert np.array_equal(u8, orc.prob_to_u8(oracle))
    assert np.all(u8 == np.uint8(round(want * 255)))
