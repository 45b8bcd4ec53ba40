"""The layer-stack (wide-ink) UNet: 4 stages of 64/128/256/512 channels whose first two strided
stages halve y and x only (stride (1, 2, 2)) and whose last halves all three axes, a one-class
sigmoid head, anisotropic z x y x x tiles.

The reference builds its UNets with one int stride per stage (src/ml/nets/resenc_unet.hpp:141-158,
168-175) and tiles cubes (src/ml/infer.hpp:39, 459); this net is nnU-Net's per-axis stride
generalisation of the same modules (ConvNormAct, ConvStack, ConvTranspose3d with kernel = stride,
a 1x1x1 head + sigmoid), so the parity reference is that network computed in fp32 by PyTorch
(tests/quant_model.py, conv3d / conv_transpose3d with stride tuples), on per-tile z-scored input
(src/ml/infer.hpp:350-385).

Bounds as everywhere: 16-bit operands max-abs <= 1e-2 against fp32; e4m3 operands against the
model with the same operand rounding (kernel parity) and Dice against fp32."""
from pathlib import Path

import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import INK_FEATURES, INK_STRIDES, make_plain_unet, plain_unet_params

pytestmark = pytest.mark.gpu

TOL16 = 1e-2
GOLD = Path(__file__).resolve().parent / "golden"


def zscore(t):
    """The reference's per-tile z-score (src/ml/infer.hpp:350-385): exact sums, double steps."""
    v = t.astype(np.float64).ravel()
    n = v.size
    S, Q = float(t.astype(np.int64).sum()), float((t.astype(np.int64) ** 2).sum())
    mean = S / n
    var = Q / n - mean * mean
    sd = np.sqrt(max(var, 1e-12))
    return ((v - mean) / sd).astype(np.float32).reshape(t.shape)


def dice(a, b):
    s = a.sum() + b.sum()
    return 1.0 if s == 0 else 2.0 * (a & b).sum() / s


def ink_tiles(shape, n, seed):
    rng = np.random.default_rng(seed)
    base = rng.normal(110, 20, size=(n,) + shape)
    base[:, :, shape[1] // 4: shape[1] // 2, shape[2] // 3: 2 * shape[2] // 3] += 25.0
    return np.clip(np.rint(base), 0, 255).astype(np.uint8)


@pytest.mark.parametrize("tile", [(16, 64, 64), (32, 64, 128)])
def test_ink_forward_f16_matches_fp32(cuda_torch, tmp_path, tile):
    torch = cuda_torch
    import quant_model as qm

    params = plain_unet_params(INK_FEATURES, ncls=1, seed=3, strides=INK_STRIDES)
    w = make_plain_unet(tmp_path / "ink.fxweights", INK_FEATURES, ncls=1, seed=3, strides=INK_STRIDES)
    net = fx.Net(w, tile, max_batch=2, precision="f16")
    assert net.patch is None and net.tile == tile
    assert net.stage_masks() == [0, 3, 3, 7]
    tiles = ink_tiles(tile, 2, 11)
    dt = torch.from_numpy(tiles).cuda()
    prob = torch.zeros((2,) + tile, device="cuda")
    net.forward_dev(dt.data_ptr(), 2, prob.data_ptr(), channel=0, sigmoid=1)
    torch.cuda.synchronize()
    got = prob.cpu()
    x = torch.from_numpy(np.stack([zscore(t) for t in tiles]))[:, None]
    with torch.no_grad():
        want = qm.forward(params, x)
    e = (got - want).abs()
    d = dice(got.numpy() >= 0.5, want.numpy() >= 0.5)
    print(f"ink {tile} f16 forward vs fp32: max-abs {e.max():.3e} mean {e.mean():.3e} Dice {d:.5f}")
    net.close()
    assert float(e.max()) <= TOL16 and d >= 0.99


def test_ink_forward_fp8_matches_quantised_model(cuda_torch, tmp_path):
    torch = cuda_torch
    import quant_model as qm

    tile = (16, 64, 64)
    params = plain_unet_params(INK_FEATURES, ncls=1, seed=3, strides=INK_STRIDES)
    w = make_plain_unet(tmp_path / "ink.fxweights", INK_FEATURES, ncls=1, seed=3, strides=INK_STRIDES)
    net = fx.Net(w, tile, max_batch=2, precision="fp8")
    net.calibrate(ink_tiles(tile, 4, 21))
    scales = dict(zip(qm.layer_keys(len(INK_FEATURES)), (float(v) for v in net.act_scales())))
    tiles = ink_tiles(tile, 2, 12)
    dt = torch.from_numpy(tiles).cuda()
    prob = torch.zeros((2,) + tile, device="cuda")
    net.forward_dev(dt.data_ptr(), 2, prob.data_ptr(), channel=0, sigmoid=1)
    torch.cuda.synchronize()
    got = prob.cpu()
    x = torch.from_numpy(np.stack([zscore(t) for t in tiles]))[:, None]
    with torch.no_grad():
        want_q = qm.forward(params, x, types=qm.gpu_types(INK_FEATURES, "fp8"), scales=scales)
        want_32 = qm.forward(params, x)
    eq, e32, em = (got - want_q).abs(), (got - want_32).abs(), (want_q - want_32).abs()
    g5, q5, f5 = got.numpy() >= 0.5, want_q.numpy() >= 0.5, want_32.numpy() >= 0.5
    dq, d32, dm = dice(g5, q5), dice(g5, f5), dice(q5, f5)
    print(f"ink fp8 forward: vs quantised model max-abs {eq.max():.2e} mean {eq.mean():.2e} Dice {dq:.5f}; "
          f"vs fp32 mean {e32.mean():.2e} Dice {d32:.5f}; model vs fp32 mean {em.mean():.2e} Dice {dm:.5f}")
    net.close()
    # kernel parity as for the surface nets: the GPU sits closer to the quantised model than the
    # format's own error, and carries that error (same distance and Dice to fp32). This random-init
    # net's sigmoid leaves much of the tile near 0.5, so the threshold flips of a different
    # summation order cost more Dice than on the surface nets' softmax maps.
    assert eq.mean() <= em.mean()
    assert abs(e32.mean() - em.mean()) <= 0.25 * em.mean()
    assert abs(d32 - dm) <= 0.01
    assert dq >= 0.95


def test_ink_tile_rejections(cuda_torch, tmp_path):
    """Extents that do not halve evenly through the stages, TTA on a non-cubic tile, and the
    cube-only entry points are refused with an error, not run."""
    w = make_plain_unet(tmp_path / "ink.fxweights", INK_FEATURES, ncls=1, seed=3, strides=INK_STRIDES)
    with pytest.raises(fx.FxError):
        fx.Net(w, (15, 64, 64), max_batch=1, precision="f16")  # the last stage halves z: 15 is odd
    net = fx.Net(w, (16, 64, 64), max_batch=1, precision="f16")
    vol = ink_tiles((16, 64, 64), 1, 5)[0]
    with pytest.raises(fx.FxError):
        net.predict_volume(vol, overlap=0.25, batch=1, sigmoid=1, channel=0, tta=8)
    net.close()


def test_ink_window_matches_oracle_map(cuda_torch, tmp_path):
    """The anisotropic sliding window (per-axis tile starts, Gaussians of sigma tile / 8, blend,
    normalisation) on a papyrus stack against the C oracle's full map (tests/golden/ink_small.npz):
    every voxel, f16 <= 1e-2 max-abs; the calibrated fp8 schedule Dice >= 0.99."""
    g = np.load(GOLD / "ink_small.npz")
    w = make_plain_unet(tmp_path / "ink.fxweights", INK_FEATURES, ncls=1, seed=int(g["weight_seed"]),
                        strides=INK_STRIDES)
    tile = tuple(int(v) for v in g["tile"])
    vol = fx.synth_papyrus(tuple(int(v) for v in g["shape"]), int(g["volume_seed"]), int(g["stack"]))
    ref = g["prob_u16"].astype(np.float32) / np.float32(65535.0)
    net = fx.Net(w, tile, max_batch=4, precision="f16")
    prob, u8 = net.predict_volume(vol, overlap=float(g["overlap"]), batch=4, channel=0, sigmoid=1)
    net.close()
    e = np.abs(prob - ref)
    d = dice(prob >= 0.5, ref >= 0.5)
    print(f"ink window f16 vs oracle: max-abs {e.max():.3e} mean {e.mean():.3e} Dice {d:.5f} over {prob.size} voxels")
    assert float(e.max()) <= TOL16 and d >= 0.99
    assert np.abs(u8.astype(int) - np.clip(np.floor(ref * 255 + 0.5), 0, 255).astype(int)).max() <= 3
    net = fx.Net(w, tile, max_batch=4, precision="fp8")
    cal = np.stack([fx.synth_papyrus(tile, 1000 + i, 0) for i in range(4)])
    dc, mc = net.calibrate_schedule(cal, min_dice=0.993)
    f8 = [l["name"] for l in net.layers() if l["precision"] == "fp8"]
    prob8, _ = net.predict_volume(vol, overlap=float(g["overlap"]), batch=4, channel=0, sigmoid=1)
    net.close()
    e8 = np.abs(prob8 - ref)
    d8 = dice(prob8 >= 0.5, ref >= 0.5)
    print(f"ink window fp8 schedule ({len(f8)} e4m3 layers {f8}, calibration Dice {dc:.5f}): vs oracle max-abs "
          f"{e8.max():.3e} mean {e8.mean():.3e} Dice {d8:.5f}")
    assert d8 >= 0.99


def test_ink_full_stack_matches_fp32(cuda_torch, tmp_path):
    """The workload's own sizes: one 64 x 512 x 512 papyrus stack in 64 x 256 x 256 tiles at
    overlap 0.25 (1 x 3 x 3 tiles). Reference = every tile through the fp32 PyTorch network on the
    GPU (TF32 off) and the per-axis Gaussian blend in float64; the f16 path must agree to 1e-2 on
    every one of the 16.8 M voxels."""
    torch = cuda_torch
    import quant_model as qm
    from oracle import oracle as orc

    tile, ov, shape = (64, 256, 256), 0.25, (64, 512, 512)
    params = plain_unet_params(INK_FEATURES, ncls=1, seed=3, strides=INK_STRIDES)
    w = make_plain_unet(tmp_path / "ink.fxweights", INK_FEATURES, ncls=1, seed=3, strides=INK_STRIDES)
    vol = fx.synth_papyrus(shape, 3, 0)
    net = fx.Net(w, tile, max_batch=2, precision="f16")
    prob, _ = net.predict_volume(vol, overlap=ov, batch=2, channel=0, sigmoid=1, want_u8=False)
    net.close()
    starts = [orc.tile_starts(shape[a], tile[a], ov) for a in range(3)]
    gw = [orc.gaussian1d(tile[a]).astype(np.float64) for a in range(3)]
    wt = gw[0][:, None, None] * gw[1][None, :, None] * gw[2][None, None, :]
    acc = np.zeros(shape, np.float64)
    wsum = np.zeros(shape, np.float64)
    old = (torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32)
    torch.backends.cudnn.allow_tf32 = torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for z0 in starts[0]:
            for y0 in starts[1]:
                for x0 in starts[2]:
                    t = vol[z0:z0 + tile[0], y0:y0 + tile[1], x0:x0 + tile[2]]
                    x = torch.from_numpy(zscore(t))[None, None].cuda()
                    with torch.no_grad():
                        p = qm.forward(params, x)[0].double().cpu().numpy()
                    acc[z0:z0 + tile[0], y0:y0 + tile[1], x0:x0 + tile[2]] += wt * p
                    wsum[z0:z0 + tile[0], y0:y0 + tile[1], x0:x0 + tile[2]] += wt
    finally:
        torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = old
    ref = acc / wsum
    e = np.abs(prob - ref)
    d = dice(prob >= 0.5, ref >= 0.5)
    print(f"ink full stack {shape} f16 vs fp32: max-abs {e.max():.3e} mean {e.mean():.3e} Dice {d:.5f}")
    assert float(e.max()) <= TOL16 and d >= 0.99


def test_ink_stacks_batch_equals_single_stacks(cuda_torch, tmp_path):
    """A batch of layer stacks in one call (fx_infer_opts.stacks) equals predicting each stack
    alone: tile starts and blend run per stack, no tile crosses a stack boundary (only the
    grouping of tiles into forwards differs). The device-resident entry point
    (fx_predict_volume_dev) equals the host one up to the order of the blend's atomic adds (up to
    eight tiles cover a voxel here, so float sums may round differently)."""
    torch = cuda_torch
    tile = (16, 64, 64)
    w = make_plain_unet(tmp_path / "ink.fxweights", INK_FEATURES, ncls=1, seed=3, strides=INK_STRIDES)
    stacks = [fx.synth_papyrus((24, 112, 96), 3, k) for k in range(3)]
    net = fx.Net(w, tile, max_batch=8, precision="f16")
    single = [net.predict_volume(v, overlap=0.25, batch=8, channel=0, sigmoid=1)[0] for v in stacks]
    vol = np.concatenate(stacks, 0)
    prob, u8 = net.predict_volume(vol, overlap=0.25, batch=8, channel=0, sigmoid=1, stacks=3)
    err = max(float(np.abs(prob[24 * k:24 * (k + 1)] - single[k]).max()) for k in range(3))
    print(f"ink stacks: batched vs single max-abs {err:.2e}")
    assert err <= 1e-3
    dv = torch.from_numpy(vol).cuda()
    dp = torch.zeros(vol.shape, dtype=torch.float32, device="cuda")
    du = torch.zeros(vol.shape, dtype=torch.uint8, device="cuda")
    net.predict_volume_dev(dv.data_ptr(), vol.shape, dp.data_ptr(), du.data_ptr(), overlap=0.25, batch=8, channel=0,
                           sigmoid=1, stacks=3, stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    fx.check(fx.lib().fx_net_device_status(net.handle))
    e_dev = float(np.abs(dp.cpu().numpy() - prob).max())
    print(f"ink stacks: device entry vs host entry max-abs {e_dev:.2e}")
    assert e_dev <= 1e-6
    assert np.abs(du.cpu().numpy().astype(int) - u8.astype(int)).max() <= 1
    with pytest.raises(fx.FxError):  # a stack thinner than the tile
        net.predict_volume(np.zeros((30, 64, 64), np.uint8), overlap=0.25, batch=2, channel=0, sigmoid=1, stacks=2)
    net.close()
