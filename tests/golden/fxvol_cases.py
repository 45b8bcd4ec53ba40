"""Inputs of the .fxvol codec fixtures: 64^3 chunks and a small volume built with integer arithmetic
only (and IEEE divisions for the f32 cases), so every machine regenerates them bit for bit.
Shared by tests/golden/make_golden.py (which runs the reference's codec on them) and the tests."""
from __future__ import annotations

import numpy as np

T = 64


def _grid(n=T, shape=None):
    shape = shape or (n, n, n)
    return np.meshgrid(*(np.arange(s, dtype=np.int64) for s in shape), indexing="ij")


def _hash(z, y, x, seed):
    h = (z * 73856093) ^ (y * 19349663) ^ (x * 83492791) ^ (seed * 2654435761)
    h = (h * 2246822519) & 0xFFFFFFFF
    h ^= h >> 13
    h = (h * 3266489917) & 0xFFFFFFFF
    h ^= h >> 16
    return h


def chunk_u8(kind: str) -> np.ndarray:
    z, y, x = _grid()
    if kind == "zeros":
        v = np.zeros_like(z)
    elif kind == "const":
        v = np.full_like(z, 200)
    elif kind == "ramp":  # a triangle wave: smooth, no wrap
        t = (z * 5 + y * 3 + x * 2 + (z * y) // 8) % 510
        v = np.where(t < 256, t, 509 - t)
    elif kind == "sphere":
        v = np.where((z - 30) ** 2 + (y - 34) ** 2 + (x - 29) ** 2 < 500, 250, 3)
    elif kind == "sheet":  # a prediction-like bright sheet with a linear falloff
        d = np.abs(z * 3 + y * 2 - x * 4 - 40) // 2
        v = np.maximum(0, 255 - d * 20)
    elif kind == "noise":
        v = _hash(z, y, x, 1) >> 24
    elif kind == "mixed":
        t = (z * 5 + y * 3 + x * 2 + (z * y) // 8) % 510
        v = np.clip(np.where(t < 256, t, 509 - t) + (_hash(z, y, x, 2) & 15) - 8, 0, 255)
    elif kind == "checker":
        v = ((z // 2 + y // 2 + x // 2) & 1) * 255
    else:
        raise KeyError(kind)
    return v.astype(np.uint8)


def chunk_f32(kind: str) -> np.ndarray:
    z, y, x = _grid()
    if kind == "f32_smooth":  # octave-pyramid-like values: means with non-dyadic fractions
        v = (z * y - (x * x) // 3 + 7 * z) / 7.0
    elif kind == "f32_signed":
        v = ((_hash(z, y, x, 3) % 60001).astype(np.int64) - 30000) / 100.0
    elif kind == "f32_zeros":
        v = np.zeros(z.shape)
    else:
        raise KeyError(kind)
    return v.astype(np.float32)


# (kind, q): every u8 kind at the prediction q = 32 and the reference default 8, the noisy ones at a
# fine q so that category planes pass 4096 symbols (the 4-state interleaved rANS)
TILE_CASES_U8 = [(k, 32.0) for k in ("zeros", "const", "ramp", "sphere", "sheet", "noise", "mixed", "checker")] + \
    [(k, 8.0) for k in ("ramp", "sphere", "sheet", "noise", "mixed")] + [("mixed", 2.0), ("checker", 4.0)]
TILE_CASES_F32 = [("f32_smooth", 32.0), ("f32_signed", 8.0), ("f32_zeros", 32.0)]

ARCHIVE_DIMS = (150, 100, 130)  # 3 x 2 x 3 chunks, ragged far faces, 3 LODs
ARCHIVE_Q = 32.0


def archive_volume() -> np.ndarray:
    """A prediction-like volume: two bright sheets with falloff in z < 128; the z >= 128 chunk row
    is empty, so those chunks are ZERO slots."""
    z, y, x = _grid(shape=ARCHIVE_DIMS)
    d1 = np.abs(z * 3 + y * 2 - x * 4 - 40) // 2
    d2 = np.abs(z * 2 - y * 3 + x - 90) // 3
    v = np.maximum(np.maximum(0, 255 - d1 * 20), np.maximum(0, 230 - d2 * 25))
    v = np.where(z < 128, v, 0)
    return v.astype(np.uint8)
