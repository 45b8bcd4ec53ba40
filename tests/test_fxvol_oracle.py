"""The .fxvol oracle pinned to the reference (CPU): the C restatement of the tile codec against the
reference's own encode_tile_dct / decode_tile_dct outputs (tests/golden/fxvol_tiles.npz), its
DCT-16 against the orthonormal DCT-II, corrupt-payload rejection (the reference's
tests/test_dct_block.cpp cases), and the library's container against an archive the reference
wrote (tests/golden/fxvol_small.fxvol): every payload rewritten through fx_fxvol_* gives the same
file byte for byte."""
import hashlib
import importlib.util
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as orc

GOLD = Path(__file__).resolve().parent / "golden"
_spec = importlib.util.spec_from_file_location("fxvol_cases", GOLD / "fxvol_cases.py")
fc = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(fc)
TILES = np.load(GOLD / "fxvol_tiles.npz")


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def cases():
    for kind, q in fc.TILE_CASES_U8:
        yield "u8", kind, q
    for kind, q in fc.TILE_CASES_F32:
        yield "f32", kind, q


def src(dtype, kind):
    return fc.chunk_u8(kind) if dtype == "u8" else fc.chunk_f32(kind)


@pytest.mark.parametrize("dtype,kind,q", list(cases()))
def test_oracle_decode_matches_reference(dtype, kind, q):
    key = f"{dtype}_{kind}_q{q:g}"
    rc, u8, f = orc.fxv_decode(TILES[f"pay_{key}"].tobytes(), q)
    assert rc == 0
    assert sha(u8) == str(TILES[f"sha_u8_{key}"])
    assert sha(f) == str(TILES[f"sha_f32_{key}"])


@pytest.mark.parametrize("dtype,kind,q", list(cases()))
def test_oracle_encode_matches_reference(dtype, kind, q):
    key = f"{dtype}_{kind}_q{q:g}"
    want = TILES[f"pay_{key}"].tobytes()
    assert orc.fxv_encode(src(dtype, kind), q, log2_mode=0) == want  # glibc log2, as the reference
    assert orc.fxv_encode(src(dtype, kind), q, log2_mode=1) == want  # the device's portable log2


def test_roundtrip_quality_bounds():
    # the reference's test_dct_block.cpp:30-58 bounds on smooth data: mean error below q, no
    # outlier beyond 12 q; a hard 3 -> 250 step and +-8 noise only keep the mean within 2 q
    for kind in ("ramp", "sheet", "sphere", "mixed"):
        for q in (4.0, 8.0, 32.0):
            t = fc.chunk_u8(kind)
            rc, u8, _ = orc.fxv_decode(orc.fxv_encode(t, q), q)
            err = np.abs(u8.astype(np.float64) - t)
            assert rc == 0, (kind, q)
            if kind in ("ramp", "sheet"):
                assert err.mean() < q and err.max() < 12 * q, (kind, q, err.mean(), err.max())
            else:
                assert err.mean() < 2 * q, (kind, q, err.mean())


def test_dct16_is_the_orthonormal_dct2():
    from scipy.fft import dctn, idctn

    rng = np.random.default_rng(3)
    b = rng.uniform(-200, 200, (16, 16, 16)).astype(np.float32)
    got = orc.fxv_dct3(b)
    want = dctn(b.astype(np.float64), type=2, norm="ortho")
    assert np.abs(got - want).max() < 2e-3
    back = orc.fxv_dct3(got, inverse=True)
    assert np.abs(back - idctn(want, type=2, norm="ortho")).max() < 2e-3
    assert np.abs(back - b).max() < 2e-3


def test_portable_log2():
    xs = np.concatenate([np.geomspace(1e-6, 1e9, 2000), np.arange(1, 300, dtype=np.float64)])
    err = max(abs(orc.lib().fxv_log2_series(float(x)) - np.log2(x)) for x in xs)
    assert err < 4e-15


def test_crc32c_and_morton():
    assert orc.lib().fxv_crc32c(b"123456789", 9) == 0xE3069283  # the CRC-32C check value
    assert orc.lib().fxv_morton3(0, 0, 1) == 1 and orc.lib().fxv_morton3(0, 1, 0) == 2
    assert orc.lib().fxv_morton3(1, 0, 0) == 4 and orc.lib().fxv_morton3(3, 5, 6) == 0b011101110


def test_oracle_rejects_corrupt_payloads():
    # test_dct_block.cpp:93-129: truncation at every length, random garbage, a corrupt K byte
    good = TILES["pay_u8_sheet_q32"].tobytes()
    for n in range(0, len(good), max(1, len(good) // 97)):
        rc, _, _ = orc.fxv_decode(good[:n], 32.0)
        assert rc != 0, n
    rng = np.random.default_rng(9)
    for _ in range(50):
        rc, _, _ = orc.fxv_decode(rng.integers(0, 256, rng.integers(1, 4000)).astype(np.uint8).tobytes(), 32.0)
    # K is the byte after the 128 DC / nsig varints; 0 and 9 are out of range
    p = 0
    for _ in range(128):
        while good[p] & 0x80:
            p += 1
        p += 1
    for k in (0, 9, 255):
        bad = bytearray(good)
        bad[p] = k
        rc, _, _ = orc.fxv_decode(bytes(bad), 32.0)
        assert rc != 0


def test_container_reader_and_rewrite_identical(tmp_path):
    import fenix_b200.fxvol as fv

    gold = GOLD / "fxvol_small.fxvol"
    meta = np.load(GOLD / "fxvol_small.npz")
    py = orc.fxvol_read_slots(gold)
    assert tuple(py["dims"]) == fc.ARCHIVE_DIMS and py["q"] == fc.ARCHIVE_Q and py["nlods"] == 3
    a = fv.VolumeArchive.open(gold)
    inf = a.info()
    assert tuple(inf.dims) == fc.ARCHIVE_DIMS and inf.nlods == 3 and inf.src_dtype == 0 and not inf.sealed
    cov = {tuple(int(v) for v in r[:4]): int(r[4]) for r in meta["coverage"]}
    assert {k: v[0] for k, v in py["slots"].items()} == cov
    assert any(v == fv.ZERO for v in cov.values()) and any(v == fv.REAL for v in cov.values())
    out = tmp_path / "rewrite.fxvol"
    b = fv.VolumeArchive.create(out, fc.ARCHIVE_DIMS, fc.ARCHIVE_Q)
    for (lod, z, y, x), c in sorted(cov.items()):
        got_cov, pay = a.chunk_payload(lod, z, y, x)
        assert got_cov == c and pay == py["slots"][(lod, z, y, x)][1]
        b.write_chunk_payload(lod, z, y, x, pay)
    b.set_nlods(inf.nlods)
    b.close()
    a.close()
    assert out.read_bytes() == gold.read_bytes()


def test_oracle_reads_reference_archive():
    meta = np.load(GOLD / "fxvol_small.npz")
    assert sha(orc.fxvol_read_u8(GOLD / "fxvol_small.fxvol")) == str(meta["sha_read"])


def test_container_rejects_corrupt_files(tmp_path):
    import fenix_b200 as fx
    import fenix_b200.fxvol as fv

    raw = (GOLD / "fxvol_small.fxvol").read_bytes()
    bad = tmp_path / "bad.fxvol"
    bad.write_bytes(raw[:5000])  # truncated below the two superblocks
    with pytest.raises(fx.FxError):
        fv.VolumeArchive.open(bad)
    b = bytearray(raw)
    for s in (0, 4096):
        b[s + 40] ^= 0xFF  # corrupt dims in both superblock copies: crc fails
    bad.write_bytes(bytes(b))
    with pytest.raises(fx.FxError):
        fv.VolumeArchive.open(bad)
    # a flipped payload byte fails the blob crc of that chunk only
    a0 = orc.fxvol_read_slots(GOLD / "fxvol_small.fxvol")
    pay = a0["slots"][(0, 0, 0, 0)][1]
    off = raw.index(pay)
    b = bytearray(raw)
    b[off + 10] ^= 0x55
    bad.write_bytes(bytes(b))
    a = fv.VolumeArchive.open(bad)
    with pytest.raises(fx.FxError):
        a.chunk_payload(0, 0, 0, 0)
    assert a.chunk_payload(0, 0, 0, 1)[0] == fv.REAL
    a.close()
