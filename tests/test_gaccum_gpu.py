"""The device GlobalAccum (fx_gaccum_*) against the reference's own GlobalAccum tests
(tests/test_global_accum.cpp: constant round trip, sweep = one shot, resume floor, untouched
chunks are zero) and a z-swept streamed prediction against the whole-volume prediction."""
import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.gaccum import GlobalAccum
from fenix_b200.weights import CONFIG1_FEATURES, make_plain_unet

pytestmark = pytest.mark.gpu


def scatter_all(acc, value):
    P = acc.patch
    sp = np.full((P, P, P), value, dtype=np.float32)
    for z0 in fx.tile_starts(acc.ext[0], P, acc.overlap):
        for y0 in fx.tile_starts(acc.ext[1], P, acc.overlap):
            for x0 in fx.tile_starts(acc.ext[2], P, acc.overlap):
                acc.scatter(acc.org[0] + z0, acc.org[1] + y0, acc.org[2] + x0, sp)


def test_constant_roundtrip(cuda_torch):
    # a full grid of constant-0.6 tiles finalises to (u8)(0.6 * 255 + 0.5) = 153 everywhere
    acc = GlobalAccum((64, 0, 64), (192, 128, 192), 64, 0.5, window_planes=192)
    scatter_all(acc, 0.6)
    out = acc.finalize_rows_below(acc.chunk_rows)
    assert out.shape == (192, 128, 192)
    want = np.uint8(np.float32(0.6) * np.float32(255.0) + np.float32(0.5))
    assert want == 153 and np.all(out == want)
    assert acc.floor_row == acc.chunk_rows


def test_sweep_equals_oneshot(cuda_torch):
    a = GlobalAccum((0, 0, 0), (192, 64, 64), 64, 0.5, window_planes=192)
    b = GlobalAccum((0, 0, 0), (192, 64, 64), 64, 0.5, window_planes=192)
    scatter_all(a, 0.25)
    scatter_all(b, 0.25)
    one = a.finalize_rows_below(a.chunk_rows)
    parts = [b.finalize_rows_below(r) for r in range(1, b.chunk_rows + 1)]
    assert all(p.shape[0] == 64 for p in parts)  # each chunk row emitted exactly once
    assert np.array_equal(np.concatenate(parts), one)
    assert b.finalize_rows_below(b.chunk_rows).shape[0] == 0  # nothing left


def test_floor_drops_below(cuda_torch):
    acc = GlobalAccum((0, 0, 0), (256, 64, 64), 64, 0.5, window_planes=128)
    acc.set_floor_row(2)  # rows 0, 1 (z < 128) finalized by an earlier run
    scatter_all(acc, 1.0)
    out = acc.finalize_rows_below(acc.chunk_rows)
    assert out.shape[0] == 128  # rows 2 and 3 only
    assert np.all(out == 255)


def test_untouched_chunk_is_zero(cuda_torch):
    acc = GlobalAccum((0, 0, 0), (64, 64, 128), 64, 0.5)
    acc.scatter(0, 0, 0, np.full((64, 64, 64), 0.5, dtype=np.float32))  # covers x < 64 only
    out = acc.finalize_rows_below(1)
    assert out.shape == (64, 64, 128)
    assert out[:, :, :64].any() and not out[:, :, 64:].any()


def test_scatter_past_window_is_refused(cuda_torch):
    acc = GlobalAccum((0, 0, 0), (256, 64, 64), 64, 0.5)  # window = 128 planes
    with pytest.raises(fx.FxError):
        acc.scatter(96, 0, 0, np.zeros((64, 64, 64), np.float32))  # reaches plane 160 > 128


def test_streamed_prediction_matches_whole_volume(cuda_torch, tmp_path):
    """predict-scroll's z-sweep: before each tile row, finalize the chunk rows it cannot touch;
    the concatenated u8 rows equal the whole-volume prediction."""
    P, ov, B = 64, 0.5, 2
    shape = (200, 96, 80)
    w = make_plain_unet(tmp_path / "c1.fxweights", CONFIG1_FEATURES, seed=0)
    vol = fx.synth_spiral(shape, 11, fx.SPIRAL_CONFIG1)
    net = fx.Net(w, P, max_batch=B, precision="f16")
    acc = GlobalAccum((0, 0, 0), shape, P, ov)  # default window: P + 64 planes
    rows = []
    for zi in range(acc.tile_rows):
        z0 = acc.row_start(zi)
        rows.append(acc.finalize_rows_below(z0 // 64))
        acc.predict_row(net, zi, vol[z0:min(z0 + P, shape[0])], batch=B)
    rows.append(acc.finalize_rows_below(acc.chunk_rows))
    got = np.concatenate(rows)
    _, want = net.predict_volume(vol, overlap=ov, batch=B)
    net.close()
    assert got.shape == want.shape
    d = np.abs(got.astype(int) - want.astype(int))
    assert d.max() <= 1 and (d > 0).mean() < 1e-3  # atomic summation order only
