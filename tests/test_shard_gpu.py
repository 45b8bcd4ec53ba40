"""z-slab sharding on two GPUs (NCCL band exchange) against the one-GPU prediction of the same
volume. Needs two devices; skipped otherwise."""
import os
import socket
import tempfile

import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import CONFIG1_FEATURES, make_plain_unet

pytestmark = pytest.mark.gpu

SHAPE, P, OV, BATCH = (160, 96, 80), 64, 0.5, 2


def _rank(rank, world, port, wpath, outdir):
    import datetime

    import torch
    import torch.distributed as dist

    from fenix_b200.shard import ShardedPredictor

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        net = fx.Net(wpath, P, max_batch=BATCH, precision="f16", device=rank)
        vol = fx.synth_spiral(SHAPE, 7, fx.SPIRAL_CONFIG1)
        sp = ShardedPredictor(net, SHAPE, OV, BATCH, rank=rank, world=world, group=dist.group.WORLD)
        me = sp.me
        host_slab = torch.from_numpy(np.ascontiguousarray(vol[me.z_lo:max(me.z_hi, me.z_lo + 1)])).pin_memory()
        host_out = torch.empty((max(me.own_hi - me.own_lo, 1),) + SHAPE[1:], dtype=torch.uint8).pin_memory()
        stream = torch.cuda.Stream()
        sp.run(host_slab=host_slab, host_out=host_out, stream=stream)
        stream.synchronize()
        np.save(os.path.join(outdir, f"r{rank}.npy"), host_out[:me.own_hi - me.own_lo].numpy())
        dist.barrier()
        net.close()
    finally:
        dist.destroy_process_group()


def test_two_gpu_shards_match_one_gpu(cuda_torch, tmp_path):
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
    net = fx.Net(w, P, max_batch=BATCH, precision="f16")
    _, want = net.predict_volume(fx.synth_spiral(SHAPE, 7, fx.SPIRAL_CONFIG1), overlap=OV, batch=BATCH)
    net.close()
    assert got.shape == want.shape
    d = np.abs(got.astype(int) - want.astype(int))
    # the band planes are summed in another order than on one GPU: u8 steps of at most 1
    assert d.max() <= 1 and (d > 0).mean() < 1e-3
