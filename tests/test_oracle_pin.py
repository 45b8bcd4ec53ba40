"""Pin the oracle (and the product's host tiling math) to the reference's own outputs.

CPU only. Golden data in tests/golden/ comes from the reference's code compiled by
oracle/Makefile (tests/golden/make_golden.py): ref_tiler_dump for the tiling math and ref_infer
(the reference's predict_surface_filled + nets::ConvStack via libtorch, fp32) for whole-volume
inference. The reference's own unit tests (tests/test_ml_tiler.cpp, test_global_accum.cpp,
test_predictions.cpp) are re-run from oracle/_ref when it has been built.
"""
import subprocess
from pathlib import Path

import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import make_plain_unet
from oracle import oracle as orc

GOLD = Path(__file__).resolve().parent / "golden"
SPIRAL_KEYS = ("pitch", "thickness", "sheet_mean", "sheet_sd", "bg_mean", "bg_sd", "blur_sigma", "speckle_sd")


@pytest.fixture(scope="module")
def tiling_gold():
    return np.load(GOLD / "tiling_ref.npz")


def _cases(gold, kind):
    for k in gold.files:
        if k.startswith(kind + "_"):
            yield k, k.split("_")[1:]


def test_tile_starts_bit_exact(tiling_gold):
    n = 0
    for k, (dim, patch, ov) in _cases(tiling_gold, "starts"):
        want = tiling_gold[k]
        for impl in (orc.tile_starts, fx.tile_starts):
            got = impl(int(dim), int(patch), float(ov))
            assert np.array_equal(got, want), (impl, k, got, want)
        n += 1
    assert n >= 10


def test_gaussian_and_profiles_bit_exact(tiling_gold):
    for k, (n,) in _cases(tiling_gold, "gauss"):
        want = tiling_gold[k]
        for impl in (orc.gaussian1d, fx.gaussian1d):
            got = impl(int(n))
            assert got.tobytes() == want.tobytes(), (impl, k)
    for k, (dim, patch, ov) in _cases(tiling_gold, "profile"):
        dim, patch, ov = int(dim), int(patch), float(ov)
        want = tiling_gold[k]
        starts = tiling_gold[f"starts_{dim}_{patch}_{ov}" if f"starts_{dim}_{patch}_{ov}" in tiling_gold.files else
                             k.replace("profile", "starts")]
        g = fx.gaussian1d(patch)
        for impl in (orc.weight_profile, fx.weight_profile):
            got = impl(g, patch, starts, 0, dim, dim)
            assert got.tobytes() == want.tobytes(), (impl, k)


# Known-answer cases restated from the reference's tests/test_ml_tiler.cpp and
# tests/test_global_accum.cpp, run against the product's host tiling.
def test_reference_known_answers():
    assert list(fx.tile_starts(64, 256, 0.5)) == [0]
    assert list(fx.tile_starts(256, 128, 0.5)) == [0, 64, 128]
    s = fx.tile_starts(300, 128, 0.5)
    assert s[-1] == 300 - 128
    for v in range(300):
        assert any(st <= v < st + 128 for st in s)
    w = fx.gaussian1d(128)
    assert w[64] >= w[0] and w[64] >= w[127] and w[0] >= 0.1 - 1e-6 and w.max() <= 1 + 1e-6 and w[64] > w[16]
    starts = fx.tile_starts(160, 64, 0.5)
    g = fx.gaussian1d(64)
    W = fx.weight_profile(g, 64, starts, 0, 160, 160)
    for c in range(160):
        ref = sum(g[c - s0] for s0 in starts if s0 <= c < s0 + 64)
        assert abs(W[c] - ref) < 1e-5


def test_crop_profile_is_a_window_of_the_global_profile():
    starts = fx.tile_starts(1000, 128, 0.25)
    g = fx.gaussian1d(128)
    full = fx.weight_profile(g, 128, starts, 0, 1000, 1000)
    part = fx.weight_profile(g, 128, starts, 300, 250, 1000)
    assert part.tobytes() == full[300:550].tobytes()


@pytest.mark.parametrize("name", ["test_ml_tiler", "test_global_accum", "test_predictions"])
def test_reference_unit_tests_pass(name):
    exe = orc.REF / name
    if not exe.exists():
        pytest.skip("oracle/_ref not built (needs the reference tree)")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr


def load_case(name, tmp_path):
    g = np.load(GOLD / f"net_{name}.npz")
    w = make_plain_unet(tmp_path / f"{name}.fxweights", tuple(int(v) for v in g["features"]),
                        seed=int(g["weight_seed"]))
    sp = dict(zip(SPIRAL_KEYS, (float(v) for v in g["spiral"])))
    vol = fx.synth_spiral(tuple(int(v) for v in g["shape"]), int(g["volume_seed"]), sp)
    return g, w, vol


@pytest.mark.parametrize("name", ["small3", "cfg1_p64", "cfg2_p64"])
def test_oracle_matches_reference_inference(name, tmp_path):
    g, w, vol = load_case(name, tmp_path)
    prob = orc.Net(w).predict_surface(vol, int(g["patch"]), float(g["overlap"]))
    got = prob.reshape(-1)[g["sample_idx"]]
    assert np.abs(got - g["sample_val"]).max() < 1e-4  # fp32 vs fp32 (observed ~1e-5)
    assert np.abs(orc.prob_to_u8(prob).astype(int) - g["u8"].astype(int)).max() <= 1
    assert abs(prob.astype(np.float64).sum() - float(g["prob_sum"])) < 1e-3 * prob.size ** 0.5


def test_oracle_zscore_matches_reference_formula():
    rng = np.random.default_rng(0)
    vol = rng.integers(0, 256, size=(40, 40, 40), dtype=np.uint8)
    t = orc.norm_tile(vol, (3, 5, 7), 32)
    x = vol[3:35, 5:37, 7:39].astype(np.float64)
    mean = x.sum() / x.size
    sd = np.sqrt(max((x * x).sum() / x.size - mean * mean, 1e-12))
    assert np.array_equal(t, ((x - mean) / sd).astype(np.float32))


def test_oracle_edge_clamp_fill():
    vol = np.arange(6 * 5 * 4, dtype=np.uint8).reshape(6, 5, 4)
    out = orc.norm_tile(vol, (0, 0, 0), 8)  # tile larger than the volume: edge-clamped reads
    raw = vol[np.minimum(np.arange(8), 5)][:, np.minimum(np.arange(8), 4)][:, :, np.minimum(np.arange(8), 3)]
    x = raw.astype(np.float64)
    mean = x.sum() / x.size
    sd = np.sqrt(max((x * x).sum() / x.size - mean * mean, 1e-12))
    assert np.array_equal(out, ((x - mean) / sd).astype(np.float32))
