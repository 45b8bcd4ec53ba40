"""z-slab sharding (fenix_b200/shard.py, fx_shard_plan) on the CPU: the rank plan, and the band fold
protocol of one pass between gloo ranks against the one-process blend of the same tiles. On the GPU
a neighbour's accumulator is read through a CUDA IPC mapping; here each rank's accumulator is a
memory-mapped file its neighbours read, with the same plan, exchanges and barriers."""
import os
import tempfile

import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.shard import exchanges, fold_bands, plan


def tile_grid(shape, P, ov):
    zs, ys, xs = (fx.tile_starts(n, P, ov) for n in shape)
    return [(int(z), int(y), int(x)) for z in zs for y in ys for x in xs]


@pytest.mark.parametrize("shape,P,ov,world", [((1024, 1024, 1024), 128, 0.5, 8), ((300, 64, 64), 64, 0.5, 3),
                                              ((64, 64, 64), 64, 0.5, 4), ((200, 96, 80), 48, 0.25, 5),
                                              ((130, 40, 40), 32, 0.5, 2)])
def test_plan_partitions_tiles_and_planes(shape, P, ov, world):
    D = shape[0]
    tiles = tile_grid(shape, P, ov)
    plans = plan(shape, P, ov, world)
    assert [p.rank for p in plans] == list(range(world))
    # tile ranges: contiguous, near-equal, covering the z-major list once
    assert plans[0].tile_begin == 0 and plans[-1].tile_end == len(tiles)
    for a, b in zip(plans, plans[1:]):
        assert a.tile_end == b.tile_begin
    sizes = [p.tile_end - p.tile_begin for p in plans]
    assert max(sizes) - min(sizes) <= 1
    live = [p for p in plans if p.tile_end > p.tile_begin]
    # owned planes partition [0, D)
    assert live[0].own_lo == 0 and live[-1].own_hi == D
    for a, b in zip(live, live[1:]):
        assert a.own_hi == b.own_lo
    for p in live:
        # the slab holds every plane the rank's tiles touch, and the planes it owns
        zs = [tiles[t][0] for t in range(p.tile_begin, p.tile_end)]
        assert p.z_lo == min(zs) and p.z_hi == min(max(zs) + P, D)
        assert p.z_lo <= p.own_lo <= p.own_hi <= p.z_hi
    # every plane some rank accumulated but does not own is sent to its owner exactly once
    ex = exchanges(plans)
    for z in range(D):
        owner = [p.rank for p in live if p.own_lo <= z < p.own_hi]
        assert len(owner) == 1
        for p in live:
            if p.z_lo <= z < p.z_hi and p.rank != owner[0]:
                assert sum(1 for s, d, z0, z1 in ex if s == p.rank and d == owner[0] and z0 <= z < z1) == 1


def fake_prob(t, o, P):
    """A deterministic per-tile 'probability' that differs between overlapping tiles."""
    g = np.indices((P, P, P)).astype(np.float64)
    v = (g[0] + o[0]) * 0.07 + (g[1] + o[1]) * 0.031 + (g[2] + o[2]) * 0.05 + t * 0.013
    return (0.5 + 0.5 * np.sin(v)).astype(np.float32)


def blend(shape, P, ov, tiles, z_lo, z_hi):
    """acc over planes [z_lo, z_hi): sum of (gz*gy)*gx*p of the given tile indices."""
    g = fx.gaussian1d(P)
    wzy = (g[:, None] * g[None, :]).astype(np.float32)
    w3 = (wzy[:, :, None] * g[None, None, :]).astype(np.float32)
    grid = tile_grid(shape, P, ov)
    acc = np.zeros((z_hi - z_lo,) + tuple(shape[1:]), np.float32)
    for t in tiles:
        z0, y0, x0 = grid[t]
        blk = (w3 * fake_prob(t, grid[t], P)).astype(np.float32)
        ez, ey, ex = min(P, shape[0] - z0), min(P, shape[1] - y0), min(P, shape[2] - x0)
        acc[z0 - z_lo:z0 - z_lo + ez, y0:y0 + ey, x0:x0 + ex] += blk[:ez, :ey, :ex]
    return acc


def finalize(acc, shape, P, ov, z_lo):
    g = fx.gaussian1d(P)
    W = [fx.weight_profile(g, P, fx.tile_starts(n, P, ov), 0, n, n) for n in shape]
    w = (W[0][z_lo:z_lo + acc.shape[0], None, None] * W[1][None, :, None]) * W[2][None, None, :]
    return np.where(w > 0, acc / np.where(w > 0, w, 1), acc).astype(np.float32)


CASE = ((150, 40, 36), 32, 0.5)


def _rank(rank, world, port, outdir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shape, P, ov = CASE
        plans = plan(shape, P, ov, world)
        me = plans[rank]
        recv = [(s, z0, z1) for s, d, z0, z1 in exchanges(plans) if d == rank]
        nz = max(me.z_hi - me.z_lo, 1)
        acc = np.lib.format.open_memmap(os.path.join(outdir, f"acc{rank}.npy"), mode="w+", dtype=np.float32,
                                        shape=(nz,) + shape[1:])
        acc[:me.z_hi - me.z_lo] = blend(shape, P, ov, range(me.tile_begin, me.tile_end), me.z_lo, me.z_hi)
        acc.flush()

        def fold(src, dz0, sz0, n):
            peer = np.load(os.path.join(outdir, f"acc{src}.npy"), mmap_mode="r")
            acc[dz0:dz0 + n] += peer[sz0:sz0 + n]

        fold_bands(me, plans, recv, dist.barrier, fold)
        own = finalize(np.asarray(acc[:me.z_hi - me.z_lo]), shape, P, ov, me.z_lo)[me.own_lo - me.z_lo:me.own_hi - me.z_lo]
        np.save(os.path.join(outdir, f"r{rank}.npy"), own)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_band_fold_matches_single_process(world):
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    shape, P, ov = CASE
    ntiles = len(tile_grid(shape, P, ov))
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(_rank, args=(world, port, td), nprocs=world, join=True)
        got = np.concatenate([np.load(os.path.join(td, f"r{r}.npy")) for r in range(world)])
    want = finalize(blend(shape, P, ov, range(ntiles), 0, shape[0]), shape, P, ov, 0)
    assert got.shape == want.shape
    # the bands' sums are added in another order than the one-process blend: float rounding only
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=1e-6)
