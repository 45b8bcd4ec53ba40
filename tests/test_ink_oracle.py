"""The layer-stack (wide-ink) workload on the checker side, without a GPU.

* Its input: papyrus layer stacks with ink (fx_synth_papyrus) equal the C oracle's restatement of
  the recipe byte for byte, carry ink on exactly floor(5% of the (y, x) columns), and have the
  recipe's texture statistics.
* Its network: the C oracle's anisotropic forward (fxo_net_forward_tiled: ConvStack with per-axis
  stride tuples, ConvTranspose3d with kernel = stride, a one-class sigmoid head) equals the same
  network computed by PyTorch in fp32 (tests/quant_model.py), and its isotropic case is the
  forward that tests/test_oracle_pin.py pins against the reference's own inference.
* Its tiling: per-axis tile starts / Gaussians of the anisotropic sliding window reduce to the
  cube rule on each axis (checked voxel for voxel against a numpy restatement on a small case)."""
import numpy as np
import pytest
import torch

import fenix_b200 as fx
from fenix_b200.weights import INK_FEATURES, INK_STRIDES, make_plain_unet, plain_unet_params
from oracle import netgen
from oracle import oracle as orc

SMALL_FEATS = (16, 32, 64)
SMALL_STRIDES = ((1, 1, 1), (1, 2, 2), (2, 2, 2))


@pytest.mark.parametrize("shape,seed,stack", [((16, 40, 56), 3, 0), ((24, 33, 47), 3, 5), ((8, 64, 64), 11, 2)])
def test_papyrus_matches_oracle(shape, seed, stack):
    assert fx.PAPYRUS_INK == orc.PAPYRUS_INK
    a, ia = fx.synth_papyrus(shape, seed, stack, want_ink=True)
    b, ib = orc.synth_papyrus(shape, seed, stack, want_ink=True)
    assert np.array_equal(a, b) and np.array_equal(ia, ib)


def test_papyrus_recipe_statistics():
    vol, ink = fx.synth_papyrus((64, 128, 128), 3, 0, want_ink=True)
    plane = 128 * 128
    assert int(ink.sum()) == int(np.floor(0.05 * plane))  # no ties among float field values
    m = ink.astype(bool)
    bg = vol[:, ~m].astype(np.float64)
    fg = vol[:, m].astype(np.float64)
    # sd 20 in the interior; the edge-clamped z taps (radius 12 of 64 layers) raise it near the ends
    assert abs(bg.mean() - 110.0) < 3.0 and 18.0 < bg.std() < 25.0
    assert abs(bg[24:40].std() - 20.0) < 2.0
    assert 20.0 < fg.mean() - bg.mean() < 30.0
    # fibre texture: correlated along z (sigma 4) far more than along x (sigma 1)
    v = vol.astype(np.float64) - vol.mean()
    cz = (v[1:] * v[:-1]).mean() / v.var()
    cx = (v[:, :, 1:] * v[:, :, :-1]).mean() / v.var()
    assert cz > 0.9 and cx < 0.8
    # a different stack of the series differs; the same one regenerates
    assert not np.array_equal(vol, fx.synth_papyrus((64, 128, 128), 3, 1))
    assert np.array_equal(vol, fx.synth_papyrus((64, 128, 128), 3, 0))


def test_ink_weights_match_product(tmp_path):
    import filecmp

    a = make_plain_unet(tmp_path / "a.fxweights", INK_FEATURES, ncls=1, seed=3, strides=INK_STRIDES)
    b = netgen.make_plain_unet(tmp_path / "b.fxweights", INK_FEATURES, ncls=1, seed=3, strides=INK_STRIDES)
    assert filecmp.cmp(a, b, shallow=False)
    w = netgen.plain_unet(INK_FEATURES, ncls=1, seed=3, strides=INK_STRIDES)
    assert w["decoder.transpconvs.0.weight"].shape == (512, 256, 2, 2, 2)
    assert w["decoder.transpconvs.2.weight"].shape == (128, 64, 1, 2, 2)


@pytest.mark.parametrize("tile", [(8, 16, 16), (4, 8, 24)])
def test_oracle_aniso_forward_matches_torch(tmp_path, tile):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    import quant_model as qm

    w = netgen.make_plain_unet(tmp_path / "s.fxweights", SMALL_FEATS, ncls=1, seed=4, strides=SMALL_STRIDES)
    params = plain_unet_params(SMALL_FEATS, ncls=1, seed=4, strides=SMALL_STRIDES)
    x = np.random.default_rng(0).normal(size=(2,) + tile).astype(np.float32)
    got = orc.Net(w).forward_tiled(x, channel=0, sigmoid=1)
    with torch.no_grad():
        want = qm.forward(params, torch.from_numpy(x)[:, None]).numpy()
    assert got.shape == want.shape
    assert np.abs(got - want).max() < 1e-5


def test_oracle_aniso_rejects_odd_tiles(tmp_path):
    w = netgen.make_plain_unet(tmp_path / "s.fxweights", SMALL_FEATS, ncls=1, seed=4, strides=SMALL_STRIDES)
    with pytest.raises(ValueError):
        orc.Net(w).forward_tiled(np.zeros((1, 3, 16, 16), np.float32), channel=0, sigmoid=1)


def test_oracle_aniso_window_matches_restatement(tmp_path):
    """fxo_predict_tiled on a small stack equals the per-axis sliding window written out in numpy
    over the oracle's own tile forward (starts, Gaussian weights, normalisation per axis)."""
    w = netgen.make_plain_unet(tmp_path / "s.fxweights", SMALL_FEATS, ncls=1, seed=4, strides=SMALL_STRIDES)
    net = orc.Net(w)
    tile, ov = (8, 16, 16), 0.25
    vol = orc.synth_papyrus((12, 28, 20), 3, 0)
    got = net.predict_tiled(vol, tile, ov, channel=0, sigmoid=1)
    starts = [orc.tile_starts(vol.shape[a], tile[a], ov) for a in range(3)]
    g = [orc.gaussian1d(tile[a]) for a in range(3)]
    acc = np.zeros(vol.shape, np.float64)
    wsum = np.zeros(vol.shape, np.float64)
    for z0 in starts[0]:
        for y0 in starts[1]:
            for x0 in starts[2]:
                idx = [np.clip(np.arange(o, o + t), 0, n - 1) for o, t, n in zip((z0, y0, x0), tile, vol.shape)]
                t = vol[np.ix_(*idx)].astype(np.float64)
                mean = t.sum() / t.size
                sd = np.sqrt(max((t ** 2).sum() / t.size - mean * mean, 1e-12))
                p = net.forward_tiled(((t - mean) / sd).astype(np.float32)[None], channel=0, sigmoid=1)[0]
                wt = g[0][:, None, None] * g[1][None, :, None] * g[2][None, None, :]
                sl = tuple(slice(o, min(o + tt, n)) for o, tt, n in zip((z0, y0, x0), tile, vol.shape))
                ext = tuple(s.stop - s.start for s in sl)
                acc[sl] += (wt * p)[: ext[0], : ext[1], : ext[2]]
                wsum[sl] += wt[: ext[0], : ext[1], : ext[2]]
    want = acc / wsum
    assert np.abs(got - want).max() < 1e-5
