"""The .fxvol archive and its chunk codec (include/fenix_b200.h fx_fxvol_*), mirroring the
reference's codec::VolumeArchive (src/codec/archive.hpp) and encode_tile_dct / decode_tile_dct
(src/codec/dct_block.hpp). Chunk decode and encode run on the GPU."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import check, lib

ABSENT, ZERO, REAL = 0, 1, 2
TILE = 64


class FxvolInfo(C.Structure):
    _fields_ = [("dims", C.c_int64 * 3), ("q", C.c_float), ("hf_exp", C.c_float), ("dz_frac", C.c_float),
                ("nlods", C.c_uint32), ("src_dtype", C.c_int32), ("sealed", C.c_int32)]


class VolumeArchive:
    """codec::VolumeArchive: ``open(path)`` read-only or ``create(path, dims, q)``."""

    def __init__(self, handle):
        self._h = handle

    @classmethod
    def open(cls, path) -> "VolumeArchive":
        h = C.c_void_p()
        check(lib().fx_fxvol_open(str(path).encode(), C.byref(h)))
        return cls(h)

    @classmethod
    def create(cls, path, dims, q: float = 8.0, src_dtype: int = 0) -> "VolumeArchive":
        h = C.c_void_p()
        dz, dy, dx = (int(v) for v in dims)
        check(lib().fx_fxvol_create(str(path).encode(), dz, dy, dx, q, src_dtype, C.byref(h)))
        return cls(h)

    def info(self) -> FxvolInfo:
        inf = FxvolInfo()
        check(lib().fx_fxvol_get_info(self._h, C.byref(inf)))
        return inf

    @property
    def dims(self) -> tuple[int, int, int]:
        return tuple(self.info().dims)

    @property
    def nlods(self) -> int:
        return self.info().nlods

    def chunk_extent(self, lod: int = 0) -> tuple[int, int, int]:
        d = list(self.dims)
        for _ in range(lod):
            d = [(v + 1) // 2 for v in d]
        return tuple((v + TILE - 1) // TILE for v in d)

    def chunk_payload(self, lod: int, cz: int, cy: int, cx: int) -> tuple[int, bytes | None]:
        cov, ptr, n = C.c_int(), C.c_void_p(), C.c_uint64()
        check(lib().fx_fxvol_chunk_payload(self._h, lod, cz, cy, cx, C.byref(cov), C.byref(ptr), C.byref(n)))
        return cov.value, (C.string_at(ptr, n.value) if cov.value == REAL else None)

    def write_chunk_payload(self, lod: int, cz: int, cy: int, cx: int, payload: bytes | None) -> None:
        buf = payload or b""
        check(lib().fx_fxvol_write_chunk_payload(self._h, lod, cz, cy, cx, buf if buf else None, len(buf)))

    def set_nlods(self, n: int) -> None:
        check(lib().fx_fxvol_set_nlods(self._h, n))

    def read_volume_u8(self, device: int = 0) -> np.ndarray:
        out = np.empty(self.dims, dtype=np.uint8)
        check(lib().fx_fxvol_read_volume_u8(self._h, device, out.ctypes.data_as(C.POINTER(C.c_uint8))))
        return out

    def write_volume_u8(self, vol: np.ndarray, device: int = 0) -> None:
        v = np.ascontiguousarray(vol, dtype=np.uint8)
        if v.shape != self.dims:
            raise ValueError("dims mismatch")
        check(lib().fx_fxvol_write_volume_u8(self._h, v.ctypes.data_as(C.POINTER(C.c_uint8)), device))

    def close(self) -> None:
        if getattr(self, "_h", None):
            h, self._h = self._h, None
            check(lib().fx_fxvol_close(h))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def decode_tiles(payloads: list[bytes], q: float, hf_exp: float = 0.65, dz_frac: float = 0.80, device: int = 0,
                 want_f32: bool = False):
    """decode_tile_dct of each payload: (n, 64, 64, 64) u8, and the f32 reconstruction if asked."""
    n = len(payloads)
    blob = b"".join(payloads)
    offs = np.zeros(n, dtype=np.uint64)
    lens = np.array([len(p) for p in payloads], dtype=np.uint32)
    if n:
        offs[1:] = np.cumsum(lens[:-1], dtype=np.uint64)
    u8 = np.zeros((n, TILE, TILE, TILE), dtype=np.uint8)
    f32 = np.zeros((n, TILE, TILE, TILE), dtype=np.float32) if want_f32 else None
    b = np.frombuffer(blob, dtype=np.uint8) if blob else np.zeros(1, dtype=np.uint8)
    check(lib().fx_fxvol_decode_tiles(b.ctypes.data, len(blob), offs.ctypes.data_as(C.POINTER(C.c_uint64)),
                                      lens.ctypes.data_as(C.POINTER(C.c_uint32)), n, q, hf_exp, dz_frac, device,
                                      u8.ctypes.data, f32.ctypes.data if f32 is not None else None))
    return (u8, f32) if want_f32 else u8


def encode_tiles(tiles: np.ndarray, q: float, hf_exp: float = 0.65, dz_frac: float = 0.80,
                 device: int = 0) -> list[bytes]:
    """encode_tile_dct of each (64, 64, 64) tile of a u8 or f32 array of shape (n, 64, 64, 64)."""
    t = np.ascontiguousarray(tiles)
    if t.dtype not in (np.uint8, np.float32) or t.shape[1:] != (TILE, TILE, TILE):
        raise ValueError("tiles must be (n, 64, 64, 64) u8 or f32")
    n = t.shape[0]
    cap = max(1 << 16, n * (TILE ** 3) * 3)
    out = np.zeros(cap, dtype=np.uint8)
    offs = np.zeros(n, dtype=np.uint64)
    lens = np.zeros(n, dtype=np.uint32)
    check(lib().fx_fxvol_encode_tiles(t.ctypes.data if t.dtype == np.uint8 else None,
                                      t.ctypes.data if t.dtype == np.float32 else None, n, q, hf_exp, dz_frac, device,
                                      out.ctypes.data, cap, offs.ctypes.data_as(C.POINTER(C.c_uint64)),
                                      lens.ctypes.data_as(C.POINTER(C.c_uint32))))
    return [out[int(o):int(o) + int(n_)].tobytes() for o, n_ in zip(offs, lens)]


def _sheets(shape) -> np.ndarray:
    """A prediction-like u8 volume: four bright planar sheets with a linear falloff, zero elsewhere."""
    z, y, x = np.meshgrid(*(np.arange(s, dtype=np.int64) for s in shape), indexing="ij")
    v = np.zeros(shape, np.int64)
    for k, (a, b, c, d) in enumerate([(3, 2, -4, 40), (2, -3, 1, 90), (1, 1, 1, 300), (5, -1, 2, 700)]):
        dist = np.abs(z * a + y * b + x * c - d - 37 * k) // (2 + k)
        v = np.maximum(v, np.maximum(0, 255 - dist * 24))
    return v.astype(np.uint8)


def _bench(argv=None) -> None:
    """python -m fenix_b200.fxvol bench [--size N] [--reps R] [--q Q] [--device D]: archive write
    (LOD 0 + pyramid) and LOD-0 read of a synthetic prediction-like N^3 volume, best of R, as JSON."""
    import argparse
    import json
    import os
    import tempfile
    import time

    ap = argparse.ArgumentParser(prog="python -m fenix_b200.fxvol bench")
    ap.add_argument("--size", type=int, default=512)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--q", type=float, default=32.0)
    ap.add_argument("--device", type=int, default=0)
    a = ap.parse_args(argv)
    vol = _sheets((a.size,) * 3)
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "v.fxvol")
        tw, tr = [], []
        for _ in range(a.reps + 1):
            t0 = time.perf_counter()
            with VolumeArchive.create(path, vol.shape, a.q) as arc:
                arc.write_volume_u8(vol, a.device)
            t1 = time.perf_counter()
            with VolumeArchive.open(path) as arc:
                back = arc.read_volume_u8(a.device)
            tr.append(time.perf_counter() - t1)
            tw.append(t1 - t0)
        size = os.path.getsize(path)
    vox = float(vol.size)
    print(json.dumps({"size": a.size, "q": a.q, "archive_bytes": size, "encode_gvox_s": vox / min(tw[1:]) / 1e9,
                      "decode_gvox_s": vox / min(tr[1:]) / 1e9,
                      "mean_abs_err": float(np.abs(back.astype(np.int32) - vol).mean())}))


if __name__ == "__main__":
    import sys

    if len(sys.argv) > 1 and sys.argv[1] == "bench":
        _bench(sys.argv[2:])
    else:
        print("usage: python -m fenix_b200.fxvol bench [--size N] [--reps R] [--q Q] [--device D]")
