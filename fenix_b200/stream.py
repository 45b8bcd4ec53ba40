"""Out-of-core sliding-window inference over several GPUs: the global tile grid of predict-scroll
(src/ml/inference.cpp:1282-1669) streamed by tile row through one device accumulator per GPU.

The reference runs one model replica per GPU on host threads that share a cursor over the tile
list and one host GlobalAccum (src/ml/inference.cpp:1402-1586, src/ml/global_accum.hpp:37-198).
Here each rank (one process per GPU) takes a contiguous range of tile rows [a, b) of the grid and
streams it: per row, fx_gaccum_predict_row copies the row's input planes from pinned host memory
and runs its tiles into the rank's window of f32 planes in HBM; fx_gaccum_finalize_below then
normalises and copies out the 64-plane chunk rows no later row of the rank reaches. Output chunk
rows are partitioned between ranks: the chunk rows a range's first two tile rows share with the
range below ([floor(z_a / 64), ceil((z_{a-1} + P) / 64))) belong to the rank below. The upper
rank copies those planes out of its window once its first two rows are in (fx_gaccum_export_planes
into a CUDA IPC buffer) and drops them without finalizing (fx_gaccum_discard_below); after every
rank has streamed its rows, each owner adds its upper neighbour's band by reading that buffer over
NVLink (fx_gaccum_add_planes, a kernel on the owner's GPU) and finalises it. Every tile row is run
exactly once and every chunk row finalised exactly once, so the result equals a one-GPU stream of
the whole grid up to the order of the band sums. The host only orders the steps (gloo barriers,
the IPC hand-over); there is no collective on the data path.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

from . import check, lib, tile_starts
from .gaccum import GlobalAccum

T = 64  # chunk edge


def row_ranges(n_rows: int, world: int) -> list[tuple[int, int]]:
    """Contiguous, near-equal tile-row ranges, at least two rows each (a range's band with the
    range below is complete after its first two rows)."""
    if world < 1 or n_rows < 2 * world:
        raise ValueError(f"stream: {n_rows} tile rows cannot give {world} ranges of at least 2 rows")
    base, extra = divmod(n_rows, world)
    out, a = [], 0
    for r in range(world):
        b = a + base + (1 if r < extra else 0)
        out.append((a, b))
        a = b
    return out


def stream_actions(zs, rows: int, P: int, D: int, rank: int, world: int) -> list[tuple]:
    """One rank's schedule over tile rows [0, rows) of a grid with row starts zs: ("row", zi),
    ("export", z0, n), ("discard", chunk_row), ("finalize", chunk_row), ("barrier",),
    ("add", z0, n), in order. Pure host logic, so the partition of rows and chunk rows between
    ranks can be checked without a GPU."""
    a, b = row_ranges(rows, world)[rank]
    ncz = (D + T - 1) // T
    lo = (zs[a] // T, -(-min(zs[a - 1] + P, D) // T)) if rank > 0 else None
    hi = (zs[b] // T, -(-min(zs[b - 1] + P, D) // T)) if rank < world - 1 else None
    band_n = lambda band: min(band[1] * T, D) - band[0] * T  # noqa: E731
    # the band is complete after the last of this rank's rows that reaches it (the second row on a
    # regular grid; a clamped last start can add one)
    last_in_band = max((zi for zi in range(a, b) if lo and zs[zi] < lo[1] * T), default=a)
    acts = []
    for zi in range(a, b):
        acts.append(("row", zi))
        if lo and zi == last_in_band:  # hand the band to the rank below, drop it here
            acts.append(("export", lo[0] * T, band_n(lo)))
            acts.append(("discard", lo[1]))
        if lo and zi < last_in_band:
            continue  # nothing of this rank below the band's end is final yet
        if zi + 1 < rows:
            lim = zs[zi + 1] // T
        else:
            lim = ncz if rows == len(zs) else zs[rows] // T
        if hi:
            lim = min(lim, hi[0])
        acts.append(("finalize", lim))
    acts.append(("barrier",))  # every band exported
    if hi:
        acts.append(("add", hi[0] * T, band_n(hi)))
        acts.append(("finalize", hi[1]))
    acts.append(("barrier",))  # every band read
    return acts


def stream_window(zs, rows: int, P: int, D: int, world: int) -> int:
    """Accumulator window (planes, a multiple of 64) every rank's schedule fits in: the largest
    span from a rank's floor to the end of a row it runs."""
    need = P
    for r in range(world):
        a = row_ranges(rows, world)[r][0]
        floor = zs[a] // T if r > 0 else 0
        for act in stream_actions(zs, rows, P, D, r, world):
            if act[0] == "row":
                need = max(need, min(zs[act[1]] + P, D) - floor * T)
            elif act[0] in ("discard", "finalize"):
                floor = max(floor, act[1])
    return -(-need // T) * T


class StreamRank:
    """One rank's share of a streamed prediction of a (D, H, W) u8 volume over tile rows [0, rows).

    net: the rank's fenix_b200.Net (cubic patch). group: a gloo process group (None for one rank).
    planes(z0, z1) returns the u8 input planes [z0, z1) as a C-contiguous array (pinned memory for
    speed); sink(z0, u8_planes) receives each finalised run of planes. rows < the grid's row count
    streams a prefix of the grid (its last chunk rows then lack the rows not run)."""

    def __init__(self, net, shape, overlap: float, batch: int, rank: int = 0, world: int = 1, group=None,
                 rows: int | None = None, channel: int = 1, sigmoid: int = 0):
        import torch

        self.torch = torch
        self.net, self.shape, self.overlap, self.batch = net, tuple(int(v) for v in shape), overlap, batch
        self.rank, self.world, self.group = rank, world, group
        self.channel, self.sigmoid = channel, sigmoid
        P = net.patch
        D, H, W = self.shape
        self.zs = [int(v) for v in tile_starts(D, P, overlap)]
        self.rows = len(self.zs) if rows is None else min(int(rows), len(self.zs))
        self.a, self.b = row_ranges(self.rows, world)[rank]
        self.ncz = (D + T - 1) // T
        zs = self.zs
        # the chunk rows shared with the range below (exported) and above (owned, imported)
        self.lo_band = (zs[self.a] // T, math.ceil(min(zs[self.a - 1] + P, D) / T)) if rank > 0 else None
        self.hi_band = ((zs[self.b] // T, math.ceil(min(zs[self.b - 1] + P, D) / T))
                        if rank < world - 1 else None)
        self.plane = H * W
        win = stream_window(zs, self.rows, P, D, world)
        self.acc = GlobalAccum((0, 0, 0), self.shape, P, overlap, window_planes=win, device=int(net.device))
        if self.lo_band:
            self.acc.set_floor_row(self.lo_band[0])
        L = lib()
        self._export_ptr = None
        self._peer = None
        if world > 1:
            import torch.distributed as dist

            handle = (C.c_uint8 * 64)()
            if self.lo_band:
                n = self._band_planes(self.lo_band)
                p = C.c_void_p()
                check(L.fx_ipc_buffer_alloc(int(net.device), max(n, 1) * self.plane * 4, C.byref(p), handle))
                self._export_ptr = p.value
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            if self.hi_band:
                p = C.c_void_p()
                check(L.fx_ipc_open(int(net.device), (C.c_uint8 * 64).from_buffer_copy(handles[rank + 1]),
                                    C.byref(p)))
                self._peer = p.value
        self.finalised = 0  # voxels finalised by this rank

    def _band_planes(self, band) -> int:
        return min(band[1] * T, self.shape[0]) - band[0] * T

    @property
    def input_planes(self) -> tuple[int, int]:
        """The input planes this rank reads: [z_a, z_{b-1} + P)."""
        return self.zs[self.a], min(self.zs[self.b - 1] + self.net.patch, self.shape[0])

    def _barrier(self):
        if self.world > 1:
            self.torch.distributed.barrier(group=self.group)

    def _finalize(self, lim: int, sink, out) -> None:
        n = C.c_int64()
        lo = self.acc.floor_row * T
        check(lib().fx_gaccum_finalize_below(self.acc._h, lim, out.ctypes.data_as(C.POINTER(C.c_uint8)), out.nbytes,
                                             C.byref(n)))
        if n.value:
            self.finalised += n.value * self.plane
            if sink is not None:
                sink(lo, out[: n.value])

    def actions(self) -> list[tuple]:
        """The rank's schedule (stream_actions for this rank)."""
        return stream_actions(self.zs, self.rows, self.net.patch, self.shape[0], self.rank, self.world)

    def run(self, planes, sink=None, out=None) -> None:
        """Stream the rank's rows, exchange the bands, finalise the rank's chunk rows."""
        P = self.net.patch
        L = lib()
        if out is None:
            out = np.empty((4 * T,) + self.shape[1:], dtype=np.uint8)
        for act in self.actions():
            kind = act[0]
            if kind == "row":
                zi = act[1]
                z0 = self.zs[zi]
                self.acc.predict_row(self.net, zi, planes(z0, min(z0 + P, self.shape[0])), batch=self.batch,
                                     channel=self.channel, sigmoid=self.sigmoid)
            elif kind == "export":
                check(L.fx_gaccum_export_planes(self.acc._h, act[1], act[2], self._export_ptr))
            elif kind == "discard":
                check(L.fx_gaccum_discard_below(self.acc._h, act[1]))
            elif kind == "finalize":
                self._finalize(act[1], sink, out)
            elif kind == "barrier":
                self._barrier()
            elif kind == "add":
                check(L.fx_gaccum_add_planes(self.acc._h, act[1], act[2], self._peer))

    def close(self) -> None:
        L = lib()
        if self._peer:
            check(L.fx_ipc_close(int(self.net.device), self._peer))
            self._peer = None
        self._barrier()
        if self._export_ptr:
            check(L.fx_ipc_buffer_free(int(self.net.device), self._export_ptr))
            self._export_ptr = None
        self.acc.close()
