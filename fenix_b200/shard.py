"""Multi-GPU sliding-window inference over one volume: z-slab sharding with a band exchange.

One process per GPU. The z-major tile list of the whole volume (the global grid of the
reference's predict-scroll, src/ml/inference.cpp:1282-1372) is split into contiguous, near-equal
ranges, one per rank, so tile coordinates and blend weights are those of a one-GPU run. Each rank
holds only the input z-slab its tiles read and an f32 accumulator over the same planes. Planes
are owned by exactly one rank (a partition of [0, D)); after its tiles are blended, each rank sends
the accumulator planes it computed for planes that another rank owns (the tile-overlap halo bands,
at most one tile deep) over NCCL point-to-point, the owner adds them (fx_accum_add) and finalises its
owned planes to probability / u8 on its own GPU (fx_accum_finalize). torch provides device memory,
streams and the process group; every compute step is a libfenix_b200 kernel.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import InferOpts, check, gaussian1d, lib, tile_starts, weight_profile


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
    D, H, W = shape
    zs, ys, xs = tile_starts(D, patch, overlap), tile_starts(H, patch, overlap), tile_starts(W, patch, overlap)
    per_row = len(ys) * len(xs)
    T = len(zs) * per_row
    out = []
    for r in range(world):
        t0, t1 = T * r // world, T * (r + 1) // world
        if t1 <= t0:  # more ranks than tiles: an empty rank keeps an empty slab
            out.append(RankPlan(r, t0, t0, 0, 0, 0, 0))
            continue
        iz0, iz1 = t0 // per_row, (t1 - 1) // per_row
        out.append(RankPlan(r, t0, t1, int(zs[iz0]), int(min(zs[iz1] + patch, D)), 0, 0))
    live = [p for p in out if p.tile_end > p.tile_begin]
    for i, p in enumerate(live):
        p.own_lo = 0 if i == 0 else p.z_lo
        p.own_hi = D if i == len(live) - 1 else live[i + 1].z_lo
    return out


def exchanges(plans: list[RankPlan]):
    """(src, dst, z0, z1): planes [z0, z1) that src accumulated and dst owns."""
    ex = []
    for a in plans:
        for b in plans:
            if a.rank == b.rank:
                continue
            z0, z1 = max(a.z_lo, b.own_lo), min(a.z_hi, b.own_hi)
            if z1 > z0:
                ex.append((a.rank, b.rank, z0, z1))
    return ex


def exchange_bands(acc, z_lo: int, send, recv, group, add) -> None:
    """Send this rank's accumulator planes that other ranks own, receive the bands it owns and
    fold them in with add(dst_view, src). acc holds planes [z_lo, z_lo + len(acc)); send is a list
    of (dst, z0, z1), recv of (src, z0, z1, buffer). Works for any torch device the process group
    supports (NCCL on GPUs, gloo on CPU tensors)."""
    import torch.distributed as dist

    ops = [dist.P2POp(dist.isend, acc[z0 - z_lo:z1 - z_lo].contiguous(), dst, group=group) for dst, z0, z1 in send]
    ops += [dist.P2POp(dist.irecv, buf, src, group=group) for src, z0, z1, buf in recv]
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    for src, z0, z1, buf in recv:
        add(acc[z0 - z_lo:z1 - z_lo], buf)


class ShardedPredictor:
    """Runs one rank's share of a sliding-window prediction of a (D, H, W) u8 volume."""

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
        dev = torch.device("cuda", torch.cuda.current_device())
        nz = max(self.me.z_hi - self.me.z_lo, 1)
        self.slab = torch.zeros((nz, H, W), dtype=torch.uint8, device=dev)
        self.acc = torch.zeros((nz, H, W), dtype=torch.float32, device=dev)
        self.u8 = torch.zeros((max(self.me.own_hi - self.me.own_lo, 1), H, W), dtype=torch.uint8, device=dev)
        self.recv = [(src, z0, z1, torch.empty((z1 - z0, H, W), dtype=torch.float32, device=dev))
                     for (src, dst, z0, z1) in self.ex if dst == rank]
        self.send = [(dst, z0, z1) for (src, dst, z0, z1) in self.ex if src == rank]
        self.stream = torch.cuda.Stream(device=dev)  # default stream for run(); never the null stream
        g = gaussian1d(net.patch)
        prof = [weight_profile(g, net.patch, tile_starts(n, net.patch, overlap), 0, n, n) for n in self.shape]
        self.wz, self.wy, self.wx = (torch.from_numpy(p).to(dev) for p in prof)

    @property
    def h2d_bytes(self) -> int:
        return int(self.slab.numel())

    @property
    def d2h_bytes(self) -> int:
        return int((self.me.own_hi - self.me.own_lo) * self.shape[1] * self.shape[2])

    def run(self, host_slab=None, host_out=None, stream=None) -> None:
        """One full pass: [H2D slab] -> tiles -> band exchange -> finalise owned planes [-> D2H]."""
        torch = self.torch
        L = lib()
        s = self.stream if stream is None else stream
        sp = s.cuda_stream
        if not sp:
            raise ValueError("ShardedPredictor.run needs a non-null CUDA stream")
        me = self.me
        D, H, W = self.shape
        with torch.cuda.stream(s):
            if host_slab is not None:
                self.slab.copy_(host_slab, non_blocking=True)
            self.acc.zero_()
            if me.tile_end > me.tile_begin:
                self.net.predict_tiles_dev(self.slab.data_ptr(), tuple(self.slab.shape), me.z_lo, D, self.overlap,
                                           self.batch, me.tile_begin, me.tile_end, self.acc.data_ptr(),
                                           channel=self.channel, sigmoid=self.sigmoid, stream=sp)
            if self.world > 1 and self.ex:
                exchange_bands(self.acc, me.z_lo, self.send, self.recv, self.group,
                               lambda dst, src: check(L.fx_accum_add(dst.data_ptr(), src.data_ptr(), src.numel(), sp)))
            n_own = me.own_hi - me.own_lo
            if n_own > 0:
                # Wz is indexed by slab-local z: start the profile at plane z_lo
                check(L.fx_accum_finalize(self.acc.data_ptr(), me.z_hi - me.z_lo, H, W, me.own_lo - me.z_lo,
                                          me.own_hi - me.z_lo, self.wz.data_ptr() + 4 * me.z_lo,
                                          self.wy.data_ptr(), self.wx.data_ptr(), None, self.u8.data_ptr(), sp))
                if host_out is not None:
                    host_out[:n_own].copy_(self.u8[:n_own], non_blocking=True)
