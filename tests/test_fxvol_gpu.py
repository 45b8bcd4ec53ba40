"""The device .fxvol codec and archive path against the reference and the oracle: decode of the
reference's payloads (u8 and f32 reconstruction bit for bit), encode (payload bytes equal to the
reference's encode_tile_dct and to the oracle), LOD-0 reads of an archive the reference wrote, a
write_volume that reproduces that archive byte for byte, corrupt payloads reported as decode errors,
and predict-surface over archives."""
import hashlib
import importlib.util
from pathlib import Path

import numpy as np
import pytest

import fenix_b200 as fx
import fenix_b200.fxvol as fv
from fenix_b200.weights import make_plain_unet
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
_spec = importlib.util.spec_from_file_location("fxvol_cases", GOLD / "fxvol_cases.py")
fc = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(fc)
TILES = np.load(GOLD / "fxvol_tiles.npz")


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def by_q(cases):
    out = {}
    for kind, q in cases:
        out.setdefault(q, []).append(kind)
    return out


def test_device_decode_matches_reference(cuda_torch):
    for dtype, cases in (("u8", fc.TILE_CASES_U8), ("f32", fc.TILE_CASES_F32)):
        for q, kinds in by_q(cases).items():
            keys = [f"{dtype}_{k}_q{q:g}" for k in kinds]
            u8, f32 = fv.decode_tiles([TILES[f"pay_{k}"].tobytes() for k in keys], q, want_f32=True)
            for i, k in enumerate(keys):
                assert sha(u8[i]) == str(TILES[f"sha_u8_{k}"]), k
                assert sha(f32[i]) == str(TILES[f"sha_f32_{k}"]), k


def test_device_encode_matches_reference(cuda_torch):
    for dtype, cases, gen in (("u8", fc.TILE_CASES_U8, fc.chunk_u8), ("f32", fc.TILE_CASES_F32, fc.chunk_f32)):
        for q, kinds in by_q(cases).items():
            got = fv.encode_tiles(np.stack([gen(k) for k in kinds]), q)
            for k, p in zip(kinds, got):
                assert p == TILES[f"pay_{dtype}_{k}_q{q:g}"].tobytes(), (dtype, k, q)


def test_device_codec_matches_oracle_on_random_tiles(cuda_torch):
    rng = np.random.default_rng(17)
    z, y, x = np.meshgrid(*(np.arange(64),) * 3, indexing="ij")
    tiles = []
    for k in range(6):
        base = 128 + 100 * np.sin(z / rng.uniform(4, 20) + k) * np.cos(y / rng.uniform(4, 20)) * np.sin(x / 9 + 1)
        tiles.append(np.clip(base + rng.normal(0, 4 * k, base.shape), 0, 255).astype(np.uint8))
    tiles = np.stack(tiles)
    for q in (1.0, 6.0, 32.0):
        pays = fv.encode_tiles(tiles, q)
        u8, f32 = fv.decode_tiles(pays, q, want_f32=True)
        for i in range(len(tiles)):
            assert pays[i] == orc.fxv_encode(tiles[i], q, log2_mode=1), (i, q)
            rc, ou8, of32 = orc.fxv_decode(pays[i], q)
            assert rc == 0 and np.array_equal(u8[i], ou8) and np.array_equal(f32[i].view(np.uint32), of32.view(np.uint32))
    ftiles = (tiles.astype(np.float32) / 3.0 - 40.0).astype(np.float32)
    pays = fv.encode_tiles(ftiles, 8.0)
    for i in range(len(ftiles)):
        assert pays[i] == orc.fxv_encode(ftiles[i], 8.0, log2_mode=1), i


def test_archive_read_matches_reference(cuda_torch):
    meta = np.load(GOLD / "fxvol_small.npz")
    with fv.VolumeArchive.open(GOLD / "fxvol_small.fxvol") as a:
        assert sha(a.read_volume_u8()) == str(meta["sha_read"])


def test_archive_write_reproduces_reference(cuda_torch, tmp_path):
    out = tmp_path / "w.fxvol"
    with fv.VolumeArchive.create(out, fc.ARCHIVE_DIMS, fc.ARCHIVE_Q) as a:
        a.write_volume_u8(fc.archive_volume())
    assert out.read_bytes() == (GOLD / "fxvol_small.fxvol").read_bytes()


def test_decode_rejects_corrupt_payloads(cuda_torch):
    good = TILES["pay_u8_sheet_q32"].tobytes()
    for n in (0, 1, 64, 130, len(good) // 2, len(good) - 1):
        with pytest.raises(fx.FxError) as e:
            fv.decode_tiles([good[:n]], 32.0)
        assert e.value.code == 5  # FX_DECODE_ERROR
    rng = np.random.default_rng(9)
    for _ in range(20):
        junk = rng.integers(0, 256, rng.integers(1, 4000)).astype(np.uint8).tobytes()
        try:
            fv.decode_tiles([junk], 32.0)
        except fx.FxError as err:
            assert err.code == 5
    p = 0
    for _ in range(128):
        while good[p] & 0x80:
            p += 1
        p += 1
    bad = bytearray(good)
    bad[p] = 9  # K out of range
    with pytest.raises(fx.FxError):
        fv.decode_tiles([bytes(bad)], 32.0)
    # the context is still usable
    u8 = fv.decode_tiles([good], 32.0)
    assert sha(u8[0]) == str(TILES["sha_u8_u8_sheet_q32"])


def test_predict_fxvol(cuda_torch, tmp_path):
    w = make_plain_unet(tmp_path / "n.fxweights", (16, 32, 64, 128), seed=3)
    vol = fx.synth_spiral((150, 96, 120), 5, fx.SPIRAL_CONFIG1)
    src = tmp_path / "in.fxvol"
    with fv.VolumeArchive.create(src, vol.shape, 8.0) as a:
        a.write_volume_u8(vol)
    with fv.VolumeArchive.open(src) as a:
        dec = a.read_volume_u8()
    assert np.array_equal(dec, orc.fxvol_read_u8(src))
    net = fx.Net(w, 64, max_batch=4, precision="f16")
    out = tmp_path / "out.fxvol"
    net.predict_fxvol(src, out, overlap=0.5, batch=4)
    _, u8 = net.predict_volume(dec, overlap=0.5, batch=4, want_prob=False)
    net.close()
    # the same prediction written through write_volume<u8> at q = 32 gives the same file
    ref = tmp_path / "ref.fxvol"
    with fv.VolumeArchive.create(ref, vol.shape, 32.0) as a:
        a.write_volume_u8(u8)
    assert out.read_bytes() == ref.read_bytes()
    with fv.VolumeArchive.open(out) as a:
        assert a.info().q == 32.0 and a.nlods == 3
        got = a.read_volume_u8()
    assert np.array_equal(got, orc.fxvol_read_u8(out))
    # a random-init net predicts a noise-like field, which q = 32 keeps only to about q on average
    assert np.abs(got.astype(int) - u8.astype(int)).mean() < 1.25 * 32.0
