"""ml::InferOptions features on the GPU against the reference's own predict_surface_filled with the
same options (tests/golden/feat_*.npz, full maps from oracle/_ref/ref_infer):

* octahedral TTA, 8 and 48 members (tta_infer_dev, src/ml/infer.hpp:393-441);
* pct_minmax and unit255 normalisation (norm_patch / pct_bounds, src/ml/infer.hpp:107-134, 350-385);
* the output core crop (src/ml/infer.hpp:69-76, 462-472, 532-543);
* the constant-input tile filter of predict-scroll (src/ml/inference.cpp:1885-1900), here the
  device-side skip_constant;
* a one-class sigmoid head.

The 16-bit path is held to the same bound as everywhere: max-abs <= 1e-2 against the reference's
fp32 map, Dice >= 0.99. The normalisation tables themselves are compared bit for bit with the C
oracle's per-voxel formula."""
import ast
from pathlib import Path

import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import make_plain_unet

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
TOL = 1e-2


def load(name, tmp_path):
    g = np.load(GOLD / f"feat_{name}.npz")
    feats = tuple(int(v) for v in g["features"])
    w = make_plain_unet(tmp_path / f"{name}.fxweights", feats, ncls=int(g["ncls"]), seed=int(g["weight_seed"]))
    vol = fx.synth_spiral(tuple(int(v) for v in g["shape"]), int(g["volume_seed"]), fx.SPIRAL_CONFIG1)
    if name == "skipconst":
        vol[:72] = 40
    ref = g["prob_u16"].astype(np.float32) / np.float32(65535.0)
    return g, w, vol, ast.literal_eval(str(g["options"])), ref


def dice(a, b):
    s = a.sum() + b.sum()
    return 1.0 if s == 0 else 2.0 * (a & b).sum() / s


@pytest.mark.parametrize("name", ["tta8", "tta48", "pct", "unit255", "core", "skipconst", "sigmoid"])
def test_option_matches_reference(cuda_torch, tmp_path, name):
    g, w, vol, opts, ref = load(name, tmp_path)
    P = int(g["patch"])
    net = fx.Net(w, P, max_batch=4, precision="f16")
    kw = {}
    if "tta" in opts:
        kw["tta"] = opts["tta"]
    if "norm" in opts:
        kw["norm"] = opts["norm"]
    if "core" in opts:
        kw["core"] = opts["core"]
    if "skipconst" in opts:
        kw["skip_constant"] = True
    if "sigmoid" in opts:
        kw["sigmoid"] = 1
        kw["channel"] = 0
    prob, u8 = net.predict_volume(vol, overlap=float(g["overlap"]), batch=4, **kw)
    net.close()
    assert prob.shape == ref.shape
    err = float(np.abs(prob - ref).max())
    d = dice(prob >= 0.5, ref >= 0.5)
    print(f"feat {name}: max-abs {err:.3e} Dice {d:.5f}")
    assert err <= TOL and d >= 0.99
    if name == "skipconst":  # planes only the skipped tiles reach stay exactly zero, as in the reference
        assert np.all(prob[:32] == 0.0) and np.all(ref[:32] == 0.0)


def test_tile_filter_callback(cuda_torch, tmp_path):
    """A caller's filter (InferOptions::tile_filter) is consulted once per tile; rejected tiles add
    nothing, so voxels only they cover finalise to 0."""
    w = make_plain_unet(tmp_path / "f.fxweights", (16, 32, 64, 128), seed=3)
    vol = fx.synth_spiral((128, 64, 96), 4, fx.SPIRAL_CONFIG1)
    seen = []

    def keep(z0, y0, x0, p):
        seen.append((z0, y0, x0))
        return z0 >= 32

    net = fx.Net(w, 64, max_batch=2, precision="f16")
    prob, _ = net.predict_volume(vol, overlap=0.5, batch=2, tile_filter=keep)
    full, _ = net.predict_volume(vol, overlap=0.5, batch=2)
    net.close()
    grid = [(z, y, x) for z in fx.tile_starts(128, 64, 0.5) for y in fx.tile_starts(64, 64, 0.5)
            for x in fx.tile_starts(96, 64, 0.5)]
    assert sorted(seen) == sorted(grid)
    assert np.all(prob[:32] == 0.0)
    assert not np.array_equal(prob[32:64], full[32:64])  # diluted where the dropped tiles overlapped
    assert np.allclose(prob[96:], full[96:], atol=1e-6)  # untouched where only kept tiles reach


def _oracle_norm_tile(tile_u8, norm):
    """The reference's norm_patch on one tile's f32 values (src/ml/infer.hpp:350-385), in numpy
    with the same float rounding steps."""
    v = tile_u8.astype(np.float32).ravel()
    if norm == "unit255":
        return v * np.float32(1.0 / 255.0)
    mn, mx = np.float32(v.min()), np.float32(v.max())
    if mx <= mn:
        lo, hi = mn, np.float32(mn + np.float32(1.0))
    else:
        inv = np.float32(np.float32(1023.0) / np.float32(mx - mn))
        bins = ((v - mn) * inv).astype(np.int64)
        h = np.bincount(bins, minlength=1024)
        n = v.size
        tlo, thi = int(0.5 / 100.0 * n), int(99.5 / 100.0 * n)
        c = np.cumsum(h)
        blo = int(np.nonzero(c <= tlo)[0].max()) if (c <= tlo).any() else 0
        bhi = int(np.nonzero(c < thi)[0].max()) if (c < thi).any() else 1023
        lo = np.float32(mn + np.float32(np.float32(blo) / inv))
        hi = np.float32(mn + np.float32(np.float32(bhi + 1) / inv))
        if hi <= lo:
            hi = np.float32(lo + np.float32(1.0))
    inv2 = np.float32(np.float32(1.0) / np.float32(hi - lo))
    return np.clip((v - lo) * inv2, np.float32(0.0), np.float32(1.0)).astype(np.float32)


@pytest.mark.parametrize("norm", ["pct_minmax", "unit255", "zscore"])
def test_norm_tables_bit_exact(cuda_torch, norm):
    """Every tile normalised on the device equals the reference's norm_patch restated with the same
    float steps, bit for bit (tiles inside, across the edge and larger than the volume, a constant
    tile, and a tile with a single outlier level)."""
    import ctypes as C

    torch = cuda_torch
    vol = fx.synth_spiral((70, 50, 90), 9)
    vol[:8, :8, :8] = 17                 # a constant corner
    vol[40, 20, 60] = 255                # an outlier level
    P = 32
    origins = np.array([[0, 0, 0], [6, 0, 26], [38, 18, 58], [50, 30, 70]], dtype=np.int64)
    dv = torch.from_numpy(vol).cuda()
    out = torch.zeros(len(origins), P, P, P, device="cuda")
    code = {"zscore": 0, "pct_minmax": 1, "unit255": 2}[norm]
    fx.check(fx.lib().fx_norm_tiles_mode(dv.data_ptr(), *vol.shape, origins.ctypes.data_as(C.POINTER(C.c_int64)),
                                         len(origins), P, code, out.data_ptr(), None))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for i, o in enumerate(origins):
        idx = [np.clip(np.arange(o[a], o[a] + P), 0, vol.shape[a] - 1) for a in range(3)]
        tile = vol[np.ix_(*idx)]
        if norm == "zscore":
            from oracle import oracle as orc

            want = orc.norm_tile(vol, tuple(o), P).ravel()
        else:
            want = _oracle_norm_tile(tile, norm)
        assert np.array_equal(got[i].ravel(), want), (norm, i)
    const = np.full((8, 8, 8), 17, np.uint8)
    dc = torch.from_numpy(const).cuda()
    out1 = torch.zeros(1, P, P, P, device="cuda")
    z = np.zeros((1, 3), np.int64)
    fx.check(fx.lib().fx_norm_tiles_mode(dc.data_ptr(), 8, 8, 8, z.ctypes.data_as(C.POINTER(C.c_int64)), 1, P, code,
                                         out1.data_ptr(), None))
    torch.cuda.synchronize()
    assert np.array_equal(out1.cpu().numpy().ravel(), _oracle_norm_tile(np.full((P, P, P), 17, np.uint8), norm)
                          if norm != "zscore" else np.zeros(P ** 3, np.float32))
