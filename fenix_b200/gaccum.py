"""GlobalAccum on the device (ctypes wrapper of the fx_gaccum_* entry points): the global tile
grid of predict-scroll with a z-sweep finalize and a resume floor, mirroring the reference's
ml::GlobalAccum (src/ml/global_accum.hpp:37-198)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import InferOpts, check, lib

T = 64  # chunk edge


class GlobalAccum:
    def __init__(self, org, ext, patch: int, overlap: float, window_planes: int = 0, device: int = 0):
        self.org = tuple(int(v) for v in org)
        self.ext = tuple(int(v) for v in ext)
        self.patch, self.overlap = patch, overlap
        o = (C.c_int64 * 3)(*self.org)
        e = (C.c_int64 * 3)(*self.ext)
        h = C.c_void_p()
        check(lib().fx_gaccum_create(o, e, patch, overlap, window_planes, device, C.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            lib().fx_gaccum_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def chunk_rows(self) -> int:
        return int(lib().fx_gaccum_chunk_rows(self._h))

    @property
    def floor_row(self) -> int:
        return int(lib().fx_gaccum_floor_row(self._h))

    @property
    def tile_rows(self) -> int:
        return int(lib().fx_gaccum_tile_rows(self._h))

    def row_start(self, zi: int) -> int:
        return int(lib().fx_gaccum_row_start(self._h, zi))

    def set_floor_row(self, r: int) -> None:
        check(lib().fx_gaccum_set_floor_row(self._h, r))

    def scatter(self, z0: int, y0: int, x0: int, prob: np.ndarray) -> None:
        p = np.ascontiguousarray(prob, dtype=np.float32)
        assert p.size == self.patch ** 3
        check(lib().fx_gaccum_scatter(self._h, z0, y0, x0, p.ctypes.data_as(C.POINTER(C.c_float))))

    def predict_row(self, net, zi: int, planes: np.ndarray, batch: int = 1, channel: int = 1, sigmoid: int = 0,
                    tta: int = 0):
        v = np.ascontiguousarray(planes, dtype=np.uint8)
        opts = InferOpts(self.patch, self.overlap, channel, sigmoid, batch, tta)
        check(lib().fx_gaccum_predict_row(self._h, net.handle, zi, v.ctypes.data_as(C.POINTER(C.c_uint8)),
                                          C.byref(opts)))

    def finalize_rows_below(self, row_lim: int) -> np.ndarray:
        """u8 planes [floor_row * 64, min(row_lim * 64, ext.z)) x ext.y x ext.x."""
        lo = self.floor_row * T
        hi = min(min(row_lim, self.chunk_rows) * T, self.ext[0])
        out = np.zeros((max(hi - lo, 0),) + self.ext[1:], dtype=np.uint8)
        n = C.c_int64()
        check(lib().fx_gaccum_finalize_below(self._h, row_lim, out.ctypes.data_as(C.POINTER(C.c_uint8)), out.nbytes,
                                             C.byref(n)))
        return out[: n.value]
