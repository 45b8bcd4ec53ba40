"""Multi-GPU sliding-window inference over one volume: z-slab sharding without a collective.

One process per GPU. The z-major tile list of the whole volume (the global grid of the
reference's predict-scroll, src/ml/inference.cpp:1282-1372) is split into contiguous, near-equal
ranges, one per rank (fx_shard_plan), so tile coordinates and blend weights are those of a one-GPU
run. Each rank holds only the input z-slab its tiles read and an f32 accumulator window over the
same planes. Planes are owned by exactly one rank (a partition of [0, D)). After every rank has
blended its tiles, each owner folds in the bands its neighbours accumulated for its planes (at most
one tile deep) with fx_accum_add reading the neighbour's accumulator straight from its HBM over
NVLink, through a CUDA IPC mapping handed over once at set-up, and finalises its owned planes to u8
on its own GPU (fx_accum_finalize). The host only orders the steps: two barriers per pass on a
host (gloo) process group. No NCCL, no collective on the data path. torch provides device memory,
streams and the host process group; every compute step is a libfenix_b200 kernel.

The same scheme runs in one process with one thread per GPU as fx_predict_volume_multi.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import InferOpts, check, gaussian1d, lib, tile_starts, weight_profile


class _Shard(C.Structure):
    _fields_ = [(k, C.c_int64) for k in ("tile_begin", "tile_end", "z_lo", "z_hi", "own_lo", "own_hi")]


@dataclass
class RankPlan:
    rank: int
    tile_begin: int
    tile_end: int
    z_lo: int      # slab planes [z_lo, z_hi) (input and accumulator)
    z_hi: int
    own_lo: int    # planes finalised by this rank [own_lo, own_hi)
    own_hi: int


def plan(shape, patch: int, overlap: float, world: int) -> list[RankPlan]:
    """The library's shard plan (fx_shard_plan)."""
    D, H, W = shape
    buf = (_Shard * world)()
    if lib().fx_shard_plan(D, H, W, patch, overlap, world, buf) != world:
        raise ValueError("fx_shard_plan: bad arguments")
    return [RankPlan(r, *(int(getattr(buf[r], k)) for k, _ in _Shard._fields_)) for r in range(world)]


def exchanges(plans: list[RankPlan]):
    """(src, dst, z0, z1): planes [z0, z1) that src accumulated and dst owns."""
    ex = []
    for a in plans:
        for b in plans:
            if a.rank == b.rank or a.tile_end <= a.tile_begin or b.tile_end <= b.tile_begin:
                continue
            z0, z1 = max(a.z_lo, b.own_lo), min(a.z_hi, b.own_hi)
            if z1 > z0:
                ex.append((a.rank, b.rank, z0, z1))
    return ex


def fold_bands(me: RankPlan, plans: list[RankPlan], recv, barrier, fold) -> None:
    """The host protocol of a pass once this rank's tiles are blended: wait until every rank's bands
    are complete, fold each band this rank owns (fold(src, dst_offset_planes, src_offset_planes,
    planes)), then wait until every rank has read what it needs, so no accumulator is cleared or
    freed while a neighbour still reads it."""
    barrier()
    for src, z0, z1 in recv:
        fold(src, z0 - me.z_lo, z0 - plans[src].z_lo, z1 - z0)
    barrier()


class _DevArray:
    """A raw device allocation seen by torch through __cuda_array_interface__ (no copy)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class ShardedPredictor:
    """Runs one rank's share of a sliding-window prediction of a (D, H, W) u8 volume.

    group: a host (gloo) process group over the ranks, used for the IPC hand-over at set-up and the
    two barriers of each pass; None when world == 1."""

    def __init__(self, net, shape, overlap: float, batch: int, rank: int = 0, world: int = 1, group=None,
                 channel: int = 1, sigmoid: int = 0):
        import torch

        self.torch = torch
        self.net = net
        self.shape = tuple(int(v) for v in shape)
        self.overlap = overlap
        self.batch = batch
        self.rank, self.world, self.group = rank, world, group
        self.channel, self.sigmoid = channel, sigmoid
        self.plans = plan(self.shape, net.patch, overlap, world)
        self.me = self.plans[rank]
        self.ex = exchanges(self.plans)
        D, H, W = self.shape
        self.plane = H * W
        self.dev_index = int(net.device)
        dev = torch.device("cuda", self.dev_index)
        nz = max(self.me.z_hi - self.me.z_lo, 1)
        self.slab = torch.zeros((nz, H, W), dtype=torch.uint8, device=dev)
        # the accumulator window: a buffer the neighbours map to read their bands
        L = lib()
        ptr, handle = C.c_void_p(), (C.c_uint8 * 64)()
        check(L.fx_ipc_buffer_alloc(self.dev_index, nz * self.plane * 4, C.byref(ptr), handle))
        self._acc_ptr = ptr.value
        self.acc = torch.as_tensor(_DevArray(self._acc_ptr, (nz, H, W), "<f4"), device=dev)
        self.u8 = torch.zeros((max(self.me.own_hi - self.me.own_lo, 1), H, W), dtype=torch.uint8, device=dev)
        self.recv = [(src, z0, z1) for (src, dst, z0, z1) in self.ex if dst == rank]
        self.peers = {}
        if world > 1:
            import torch.distributed as dist

            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            for src in sorted({s for s, _, _ in self.recv}):
                p = C.c_void_p()
                h = (C.c_uint8 * 64).from_buffer_copy(handles[src])
                check(L.fx_ipc_open(self.dev_index, h, C.byref(p)))
                self.peers[src] = p.value
        self.stream = torch.cuda.Stream(device=dev)  # default stream for run(); never the null stream
        g = gaussian1d(net.patch)
        prof = [weight_profile(g, net.patch, tile_starts(n, net.patch, overlap), 0, n, n) for n in self.shape]
        self.wz, self.wy, self.wx = (torch.from_numpy(p).to(dev) for p in prof)

    @property
    def h2d_bytes(self) -> int:
        return int(max(self.me.z_hi - self.me.z_lo, 0) * self.plane)

    @property
    def d2h_bytes(self) -> int:
        return int((self.me.own_hi - self.me.own_lo) * self.plane)

    @property
    def band_bytes(self) -> int:
        """Accumulator bytes this rank reads from its neighbours per pass (over NVLink)."""
        return int(sum((z1 - z0) * self.plane * 4 for _, z0, z1 in self.recv))

    def _barrier(self):
        if self.world > 1:
            self.torch.distributed.barrier(group=self.group)

    def run(self, host_slab=None, host_out=None, stream=None) -> None:
        """One full pass: [H2D slab] -> tiles -> barrier -> fold the neighbours' bands over NVLink ->
        barrier -> finalise owned planes [-> D2H]."""
        torch = self.torch
        L = lib()
        s = self.stream if stream is None else stream
        sp = s.cuda_stream
        if not sp:
            raise ValueError("ShardedPredictor.run needs a non-null CUDA stream")
        me = self.me
        D, H, W = self.shape
        live = me.tile_end > me.tile_begin
        with torch.cuda.stream(s):
            if host_slab is not None and live:
                self.slab.copy_(host_slab, non_blocking=True)
            self.acc.zero_()
            if live:
                self.net.predict_tiles_dev(self.slab.data_ptr(), tuple(self.slab.shape), me.z_lo, D, self.overlap,
                                           self.batch, me.tile_begin, me.tile_end, self.acc.data_ptr(),
                                           channel=self.channel, sigmoid=self.sigmoid, stream=sp)
        if self.world > 1:
            s.synchronize()
            check(L.fx_net_device_status(self.net.handle))
            pb = self.plane * 4

            def fold(src, dz0, sz0, nzb):
                check(L.fx_accum_add(self._acc_ptr + dz0 * pb, self.peers[src] + sz0 * pb, nzb * self.plane, sp))

            fold_bands(me, self.plans, self.recv, self._barrier, fold)
            s.synchronize()
        n_own = me.own_hi - me.own_lo
        if n_own > 0:
            with torch.cuda.stream(s):
                # Wz is indexed by slab-local z: start the profile at plane z_lo
                check(L.fx_accum_finalize(self._acc_ptr, me.z_hi - me.z_lo, H, W, me.own_lo - me.z_lo,
                                          me.own_hi - me.z_lo, self.wz.data_ptr() + 4 * me.z_lo,
                                          self.wy.data_ptr(), self.wx.data_ptr(), None, self.u8.data_ptr(), sp))
                if host_out is not None:
                    host_out[:n_own].copy_(self.u8[:n_own], non_blocking=True)

    def close(self) -> None:
        """Unmap the neighbours' buffers, wait until every rank has, then free this rank's."""
        L = lib()
        if getattr(self, "_acc_ptr", None) is None:
            return
        self.torch.cuda.synchronize(self.dev_index)
        for p in self.peers.values():
            check(L.fx_ipc_close(self.dev_index, p))
        self.peers = {}
        self._barrier()
        self.acc = None
        check(L.fx_ipc_buffer_free(self.dev_index, self._acc_ptr))
        self._acc_ptr = None
