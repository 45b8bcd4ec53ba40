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
import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import INK_FEATURES, INK_STRIDES, make_plain_unet, plain_unet_params

pytestmark = pytest.mark.gpu

TOL16 = 1e-2


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
