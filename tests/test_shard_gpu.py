"""z-slab sharding on two GPUs against the one-GPU prediction of the same volume, both ways it runs:
one process per GPU (fenix_b200.shard.ShardedPredictor: bands read from the neighbour's HBM through
a CUDA IPC mapping, host barriers on a gloo group, no NCCL) and one process with a thread per GPU
(fx_predict_volume_multi, bands read through peer mappings). Needs two devices, skipped otherwise;
the same drivers with their ranks / shards sharing one device run on one.
NVLS is off in every library the ranks use (NCCL_NVLS_ENABLE=0); the path itself uses no NCCL."""
import ctypes as C
import os
import socket
import tempfile

import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import CONFIG1_FEATURES, make_plain_unet

pytestmark = pytest.mark.gpu

SHAPE, P, OV, BATCH = (160, 96, 80), 64, 0.5, 2


def _rank(rank, world, port, wpath, outdir, one_device=False):
    import datetime

    import torch
    import torch.distributed as dist

    from fenix_b200.shard import ShardedPredictor

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = 0 if one_device else rank
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        net = fx.Net(wpath, P, max_batch=BATCH, precision="f16", device=dev)
        vol = fx.synth_spiral(SHAPE, 7, fx.SPIRAL_CONFIG1)
        sp = ShardedPredictor(net, SHAPE, OV, BATCH, rank=rank, world=world, group=dist.group.WORLD)
        me = sp.me
        host_slab = torch.from_numpy(np.ascontiguousarray(vol[me.z_lo:max(me.z_hi, me.z_lo + 1)])).pin_memory()
        host_out = torch.empty((max(me.own_hi - me.own_lo, 1),) + SHAPE[1:], dtype=torch.uint8).pin_memory()
        stream = torch.cuda.Stream()
        for _ in range(2):  # a second pass reuses the mappings and clears the accumulator
            sp.run(host_slab=host_slab, host_out=host_out, stream=stream)
            stream.synchronize()
        np.save(os.path.join(outdir, f"r{rank}.npy"), host_out[:me.own_hi - me.own_lo].numpy())
        sp.close()
        net.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def one_gpu(w):
    net = fx.Net(w, P, max_batch=BATCH, precision="f16")
    _, want = net.predict_volume(fx.synth_spiral(SHAPE, 7, fx.SPIRAL_CONFIG1), overlap=OV, batch=BATCH)
    net.close()
    return want


def close_to(got, want):
    assert got.shape == want.shape
    d = np.abs(got.astype(int) - want.astype(int))
    # the band planes are summed in another order than on one GPU: u8 steps of at most 1
    assert d.max() <= 1 and (d > 0).mean() < 1e-3


def test_two_gpu_processes_match_one_gpu(cuda_torch, tmp_path):
    torch = cuda_torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    w = make_plain_unet(tmp_path / "c1.fxweights", CONFIG1_FEATURES, seed=0)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(_rank, args=(2, port, str(w), td), nprocs=2, join=True)
        got = np.concatenate([np.load(os.path.join(td, f"r{r}.npy")) for r in range(2)])
    close_to(got, one_gpu(w))


def test_two_processes_on_one_gpu_match_one_gpu(cuda_torch, tmp_path):
    """The one-process-per-GPU driver's IPC hand-over, barriers and band fold with both ranks on one
    device (host barriers only: no kernel waits on another rank's)."""
    import torch.multiprocessing as mp

    w = make_plain_unet(tmp_path / "c1.fxweights", CONFIG1_FEATURES, seed=0)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(_rank, args=(2, port, str(w), td, True), nprocs=2, join=True)
        got = np.concatenate([np.load(os.path.join(td, f"r{r}.npy")) for r in range(2)])
    close_to(got, one_gpu(w))


def test_two_gpu_threads_match_one_gpu(cuda_torch, tmp_path):
    torch = cuda_torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    w = make_plain_unet(tmp_path / "c1.fxweights", CONFIG1_FEATURES, seed=0)
    nets = [fx.Net(w, P, max_batch=BATCH, precision="f16", device=d) for d in range(2)]
    vol = fx.synth_spiral(SHAPE, 7, fx.SPIRAL_CONFIG1)
    got = np.zeros(SHAPE, np.uint8)
    handles = (C.c_void_p * 2)(*[n.handle.value for n in nets])
    opts = fx.InferOpts(P, OV, 1, 0, BATCH, 0)
    fx.check(fx.lib().fx_predict_volume_multi(handles, 2, vol.ctypes.data_as(C.POINTER(C.c_uint8)), *SHAPE,
                                              C.byref(opts), None, got.ctypes.data_as(C.POINTER(C.c_uint8))))
    for n in nets:
        n.close()
    close_to(got, one_gpu(w))


def test_three_shards_on_one_gpu_match_one_gpu(cuda_torch, tmp_path):
    """The threaded driver's plan, band fold and owned-plane finalise with three shards sharing one
    device (each net on its own stream; the host orders the steps, nothing waits on the device)."""
    w = make_plain_unet(tmp_path / "c1.fxweights", CONFIG1_FEATURES, seed=0)
    nets = [fx.Net(w, P, max_batch=BATCH, precision="f16", device=0) for _ in range(3)]
    vol = fx.synth_spiral(SHAPE, 7, fx.SPIRAL_CONFIG1)
    got = np.zeros(SHAPE, np.uint8)
    prob = np.zeros(SHAPE, np.float32)
    handles = (C.c_void_p * 3)(*[n.handle.value for n in nets])
    opts = fx.InferOpts(P, OV, 1, 0, BATCH, 0)
    fx.check(fx.lib().fx_predict_volume_multi(handles, 3, vol.ctypes.data_as(C.POINTER(C.c_uint8)), *SHAPE,
                                              C.byref(opts), prob.ctypes.data_as(C.POINTER(C.c_float)),
                                              got.ctypes.data_as(C.POINTER(C.c_uint8))))
    for n in nets:
        n.close()
    net = fx.Net(w, P, max_batch=BATCH, precision="f16")
    want_p, want = net.predict_volume(vol, overlap=OV, batch=BATCH)
    net.close()
    close_to(got, want)
    assert float(np.abs(prob - want_p).max()) <= 1e-5
