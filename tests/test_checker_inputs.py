"""The checker side makes the benchmark's inputs without the product library (the reference arm of
bench.py and the fixture scripts use it): its synthetic volumes and network files must be the
product's, byte for byte."""
import filecmp

import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import make_plain_unet
from oracle import netgen
from oracle import oracle as orc


@pytest.mark.parametrize("shape,seed,cfg,zb,ze", [
    ((64, 50, 70), 3, "1", 0, None),
    ((96, 80, 90), 2, "3", 10, 77),
    ((40, 33, 47), 9, "3", 0, 40),
])
def test_synth_matches_product(shape, seed, cfg, zb, ze):
    sp_p = fx.SPIRAL_CONFIG1 if cfg == "1" else fx.SPIRAL_CONFIG3
    sp_o = orc.SPIRAL_CONFIG1 if cfg == "1" else orc.SPIRAL_CONFIG3
    assert sp_p == sp_o
    assert np.array_equal(fx.synth_spiral(shape, seed, sp_p, zb, ze), orc.synth_spiral(shape, seed, sp_o, zb, ze))


@pytest.mark.parametrize("features,seed", [((16, 32, 64, 128), 0), ((32, 64, 128, 256, 320), 1)])
def test_weights_match_product(tmp_path, features, seed):
    a = make_plain_unet(tmp_path / "a.fxweights", features, seed=seed)
    b = netgen.make_plain_unet(tmp_path / "b.fxweights", features, seed=seed)
    assert filecmp.cmp(a, b, shallow=False)


def test_tile_starts_match_product():
    for dim, P, ov in ((1024, 128, 0.5), (256, 128, 0.5), (192, 128, 0.5), (300, 128, 0.25), (64, 128, 0.5)):
        assert np.array_equal(fx.tile_starts(dim, P, ov), orc.tile_starts(dim, P, ov))


@pytest.mark.parametrize("shape,seed,cfg,zb,ze", [((130, 70, 150), 4, "5", 0, None), ((100, 129, 64), 4, "3", 37, 99)])
def test_chunked_synth_matches_product(shape, seed, cfg, zb, ze):
    """The out-of-core workload's generator (noise keyed per 64^3 chunk) equals the checker's, and
    any z-range regenerates the same bytes as the whole volume."""
    sp_p = fx.SPIRAL_CONFIG5 if cfg == "5" else fx.SPIRAL_CONFIG3
    sp_o = orc.SPIRAL_CONFIG5 if cfg == "5" else orc.SPIRAL_CONFIG3
    assert sp_p == sp_o
    a = fx.synth_spiral(shape, seed, sp_p, zb, ze, chunked=True)
    assert np.array_equal(a, orc.synth_spiral(shape, seed, sp_o, zb, ze, chunked=True))
    full = fx.synth_spiral(shape, seed, sp_p, chunked=True)
    assert np.array_equal(a, full[zb:ze])
    assert not np.array_equal(full, fx.synth_spiral(shape, seed, sp_p))  # a different keying
