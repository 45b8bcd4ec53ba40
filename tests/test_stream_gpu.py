"""The streamed (out-of-core) prediction on the GPU (fenix_b200/stream.py): one rank streaming the
whole tile grid row by row through the device accumulator equals fx_predict_volume over the same
global grid, and two ranks (two processes on one GPU: host barriers only, no kernel waits on
another) composing their row ranges through the IPC band exchange equal one rank. Equal up to the
order of the blend sums: u8 within one level."""
import os
import socket

import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import make_plain_unet

pytestmark = pytest.mark.gpu

SHAPE, P, OV = (448, 96, 128), 64, 0.5


def _stream(rank, world, wpath, port, out_dir, rows):
    import torch
    import torch.distributed as dist

    from fenix_b200.stream import StreamRank

    torch.cuda.set_device(0)
    group = None
    if world > 1:
        import datetime

        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
        group = dist.group.WORLD
    vol = fx.synth_spiral(SHAPE, 5, fx.SPIRAL_CONFIG1, chunked=True)
    net = fx.Net(wpath, P, max_batch=4, precision="f16")
    sr = StreamRank(net, SHAPE, OV, 4, rank=rank, world=world, group=group, rows=rows)
    res = np.zeros(SHAPE, np.uint8)
    got = np.zeros(SHAPE[0], bool)

    def sink(z0, planes):
        res[z0:z0 + len(planes)] = planes
        got[z0:z0 + len(planes)] = True

    sr.run(lambda a, b: np.ascontiguousarray(vol[a:b]), sink=sink)
    sr.close()
    net.close()
    np.save(os.path.join(out_dir, f"r{rank}.npy"), res)
    np.save(os.path.join(out_dir, f"g{rank}.npy"), got)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_stream_one_rank_equals_whole_volume(cuda_torch, tmp_path):
    w = make_plain_unet(tmp_path / "w.fxweights", (16, 32, 64, 128), seed=2)
    _stream(0, 1, str(w), 0, str(tmp_path), None)
    res, got = np.load(tmp_path / "r0.npy"), np.load(tmp_path / "g0.npy")
    assert got.all()
    vol = fx.synth_spiral(SHAPE, 5, fx.SPIRAL_CONFIG1, chunked=True)
    net = fx.Net(w, P, max_batch=4, precision="f16")
    _, want = net.predict_volume(vol, overlap=OV, batch=4)
    net.close()
    d = np.abs(res.astype(int) - want.astype(int))
    print(f"stream x1 vs fx_predict_volume: u8 max diff {d.max()}, {np.count_nonzero(d)} voxels differ")
    assert d.max() <= 1


def test_stream_two_ranks_compose(cuda_torch, tmp_path):
    import torch.multiprocessing as mp

    w = make_plain_unet(tmp_path / "w.fxweights", (16, 32, 64, 128), seed=2)
    one = tmp_path / "one"
    two = tmp_path / "two"
    one.mkdir()
    two.mkdir()
    _stream(0, 1, str(w), 0, str(one), None)
    mp.start_processes(_stream, args=(2, str(w), _free_port(), str(two), None), nprocs=2, join=True,
                       start_method="spawn")
    ref = np.load(one / "r0.npy")
    g0, g1 = np.load(two / "g0.npy"), np.load(two / "g1.npy")
    assert not (g0 & g1).any() and (g0 | g1).all()  # every plane finalised by exactly one rank
    comp = np.where(g0[:, None, None], np.load(two / "r0.npy"), np.load(two / "r1.npy"))
    d = np.abs(comp.astype(int) - ref.astype(int))
    print(f"stream x2 vs x1: u8 max diff {d.max()}, {np.count_nonzero(d)} voxels differ")
    assert d.max() <= 1 and np.count_nonzero(d) <= comp.size // 1000
