"""Residual-encoder UNet (nets::ResEncUNet: stem, BasicBlockD stages with projection / average-pool
skips, optional scSE) on the GPU against the reference's own module run on the CPU (golden
fixtures from tests/golden/make_golden.py)."""
from pathlib import Path

import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import make_resenc_unet
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"


def dice(a, b):
    a, b = a.astype(bool), b.astype(bool)
    s = a.sum() + b.sum()
    return 1.0 if s == 0 else 2.0 * (a & b).sum() / s


def load(name, tmp_path):
    g = np.load(GOLD / f"resenc_{name}.npz")
    w = make_resenc_unet(tmp_path / f"{name}.fxweights", tuple(int(v) for v in g["features"]),
                         tuple(int(v) for v in g["blocks"]), ncls=2, se=bool(g["se"]),
                         plain_naming=bool(g["plain_naming"]), seed=int(g["weight_seed"]))
    vol = fx.synth_spiral(tuple(int(v) for v in g["shape"]), int(g["volume_seed"]), fx.SPIRAL_CONFIG1)
    return g, w, vol


@pytest.mark.parametrize("name", ["plain", "scse"])
def test_resenc_f16_matches_reference(cuda_torch, tmp_path, name):
    g, w, vol = load(name, tmp_path)
    net = fx.Net(w, int(g["patch"]), max_batch=2, precision="f16")
    prob, u8 = net.predict_volume(vol, overlap=float(g["overlap"]), batch=2)
    net.close()
    err = float(np.abs(prob.reshape(-1)[g["sample_idx"]] - g["sample_val"]).max())
    du8 = int(np.abs(u8.astype(int) - g["u8"].astype(int)).max())
    d = dice(u8 >= 128, g["u8"] >= 128)
    print(f"resenc {name} f16 vs reference: sample max-abs {err:.2e}, u8 max diff {du8}, Dice {d:.5f}")
    assert err <= 1e-2 and du8 <= 4 and d >= 0.99
    assert np.array_equal(u8, orc.prob_to_u8(prob))


def test_resenc_fp8_runs_calibrated(cuda_torch, tmp_path):
    g, w, vol = load("plain", tmp_path)
    P = int(g["patch"])
    net = fx.Net(w, P, max_batch=2, precision="fp8")
    net.calibrate(np.stack([fx.synth_spiral((P, P, P), 300 + i, fx.SPIRAL_CONFIG1) for i in range(2)]))
    scales = net.act_scales()
    assert np.all(np.isfinite(scales)) and np.all(scales > 0)
    _, u8 = net.predict_volume(vol, overlap=float(g["overlap"]), batch=2)
    net.close()
    d = dice(u8 >= 128, g["u8"] >= 128)
    print(f"resenc plain fp8 vs reference: Dice {d:.5f} (e4m3 quantisation)")
    assert d >= 0.9


def test_resenc_ink_task_head_matches_reference(cuda_torch, tmp_path):
    """The reference's ink checkpoint layout (shared_encoder / shared_decoder / task_heads.ink, one
    class) under predict-ink's options (sigmoid, percentile min-max) against the reference's own
    inference (tests/golden/resenc_ink.npz)."""
    g = np.load(GOLD / "resenc_ink.npz")
    w = make_resenc_unet(tmp_path / "ink.fxweights", tuple(int(v) for v in g["features"]),
                         tuple(int(v) for v in g["blocks"]), ncls=1, se=False, plain_naming=False,
                         seed=int(g["weight_seed"]), task="ink", task_head=True)
    vol = fx.synth_papyrus(tuple(int(v) for v in g["shape"]), int(g["volume_seed"]), int(g["stack"]))
    want = g["prob_u16"].astype(np.float64) / 65535.0
    net = fx.Net(w, int(g["patch"]), max_batch=2, precision="f16")
    assert net.classes == 1
    prob, u8 = net.predict_volume(vol, overlap=float(g["overlap"]), batch=2, channel=0, sigmoid=1, norm="pct_minmax")
    net.close()
    err = float(np.abs(prob - want).max())
    d = dice(prob > 0.5, want > 0.5)
    print(f"resenc ink task head f16 vs reference: max-abs {err:.2e}, Dice {d:.5f}")
    assert err <= 1e-2 and d >= 0.99
    assert np.array_equal(u8, orc.prob_to_u8(prob))
