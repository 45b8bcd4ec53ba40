"""Resumable prediction (InferOptions::ckpt_path, src/ml/infer.hpp:136-344, 571-861): a checkpoint
in the reference's FXICKPT3 layout — written here byte for byte as the reference's CkptHeader +
u16 payload from a partial run — is resumed, the result equals an uninterrupted run to the
checkpoint's u16 quantisation, a checkpoint of another run (different overlap or weights identity)
is ignored, and the file is removed on success."""
import struct

import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import CONFIG1_FEATURES, make_plain_unet

pytestmark = pytest.mark.gpu

HDR = struct.Struct("<8s6q2Q2d5i4x")  # the reference's CkptHeader: 112 bytes


def header(dims, patch, overlap, total, done, wh, ih, scale, tta=0, channel=1, sigmoid=0, norm=0):
    return HDR.pack(b"FXICKPT3", *dims, 0, total, done, wh, ih, overlap, scale, patch, tta, channel, sigmoid, norm)


def partial_acc(torch, net, vol, P, ov, batch, k):
    """The un-normalised accumulator after the first k tiles (z-major), on the host."""
    dv = torch.from_numpy(vol).cuda()
    acc = torch.zeros(vol.shape, dtype=torch.float32, device="cuda")
    net.predict_tiles_dev(dv.data_ptr(), vol.shape, 0, vol.shape[0], ov, batch, 0, k, acc.data_ptr(),
                          stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return acc.cpu().numpy()


def weight_volume(shape, P, ov):
    w = [fx.weight_profile(fx.gaussian1d(P), P, fx.tile_starts(n, P, ov), 0, n, n) for n in shape]
    return w[0][:, None, None] * w[1][None, :, None] * w[2][None, None, :]


def test_resume_from_reference_layout_checkpoint(cuda_torch, tmp_path):
    torch = cuda_torch
    assert HDR.size == 112
    P, ov, batch = 64, 0.5, 2
    w = make_plain_unet(tmp_path / "c1.fxweights", CONFIG1_FEATURES, seed=0)
    vol = fx.synth_spiral((128, 96, 160), 7, fx.SPIRAL_CONFIG1)
    net = fx.Net(w, P, max_batch=batch, precision="f16")
    full, _ = net.predict_volume(vol, overlap=ov, batch=batch)
    total = int(np.prod([len(fx.tile_starts(n, P, ov)) for n in vol.shape]))
    k = 10
    acc = partial_acc(torch, net, vol, P, ov, batch, k)
    scale = float(acc.max())
    q = (acc * np.float32(65535.0 / scale) + np.float32(0.5)).astype(np.uint16)
    ck = tmp_path / "run.ckpt"
    ck.write_bytes(header(vol.shape, P, ov, total, k, 11, 22, scale) + q.tobytes())
    got, _ = net.predict_volume(vol, overlap=ov, batch=batch, ckpt_path=ck, ckpt_every=4, weights_hash=11,
                                input_hash=22)
    assert not ck.exists() and not (tmp_path / "run.ckpt.tmp").exists()
    # the resumed accumulator differs from the uninterrupted one by the u16 rounding of the loaded
    # part: |d acc| <= scale / 65535 / 2, so |d prob| * W stays within it
    err = np.abs(got.astype(np.float64) - full) * weight_volume(vol.shape, P, ov)
    print(f"ckpt resume: max |dp| W {err.max():.3e} (bound {scale / 65535 / 2:.3e}), max |dp| "
          f"{np.abs(got - full).max():.3e}")
    assert err.max() <= scale / 65535 / 2 + 1e-6
    a, b = got >= 0.5, full >= 0.5
    assert 2 * (a & b).sum() / (a.sum() + b.sum()) >= 0.999
    # a checkpoint of another run is ignored: start fresh, same as no checkpoint
    for bad in (header(vol.shape, P, 0.25, total, k, 11, 22, scale), header(vol.shape, P, ov, total, k, 12, 22, scale)):
        ck.write_bytes(bad + q.tobytes())
        again, _ = net.predict_volume(vol, overlap=ov, batch=batch, ckpt_path=ck, ckpt_every=4, weights_hash=11,
                                      input_hash=22)
        assert np.abs(again - full).max() <= 1e-6
        assert not ck.exists()
    # truncated payload: ignored
    ck.write_bytes(header(vol.shape, P, ov, total, k, 11, 22, scale) + q.tobytes()[:1000])
    again, _ = net.predict_volume(vol, overlap=ov, batch=batch, ckpt_path=ck, weights_hash=11, input_hash=22)
    assert np.abs(again - full).max() <= 1e-6
    # no file at all: a plain run that saves along the way and removes its file at the end
    again, _ = net.predict_volume(vol, overlap=ov, batch=batch, ckpt_path=ck, ckpt_every=2)
    assert np.abs(again - full).max() <= 1e-6 and not ck.exists()
    with pytest.raises(fx.FxError):  # checkpoints take no output crop (src/ml/infer.hpp:575)
        net.predict_volume(vol, overlap=ov, batch=batch, ckpt_path=ck, core=(8, 8, 8, 32, 32, 32))
    net.close()


def test_resume_reference_written_checkpoint(cuda_torch, tmp_path):
    """A checkpoint the reference itself wrote (tests/golden/ckpt_ref.npz: predict_surface_filled
    interrupted by its filler after 3 patches, progress saved by its own CkptWriter) is resumed by
    the GPU path, which finishes the run; the result matches the reference's uninterrupted map at
    the f16 path's bound."""
    from pathlib import Path

    g = np.load(Path(__file__).resolve().parent / "golden" / "ckpt_ref.npz")
    raw = g["ckpt"].tobytes()
    f = HDR.unpack(raw[:112])
    done, total = f[6], f[5]
    assert f[0] == b"FXICKPT3" and 0 < done < total
    w = make_plain_unet(tmp_path / "w.fxweights", tuple(int(v) for v in g["features"]), seed=int(g["weight_seed"]))
    vol = fx.synth_spiral(tuple(int(v) for v in g["shape"]), int(g["volume_seed"]), fx.SPIRAL_CONFIG1)
    ck = tmp_path / "ref.ckpt"
    ck.write_bytes(raw)
    P, ov, batch = int(g["patch"]), float(g["overlap"]), int(g["batch"])
    net = fx.Net(w, P, max_batch=batch, precision="f16")
    got, _ = net.predict_volume(vol, overlap=ov, batch=batch, ckpt_path=ck, weights_hash=int(g["whash"]),
                                input_hash=int(g["ihash"]))
    own, _ = net.predict_volume(vol, overlap=ov, batch=batch)
    net.close()
    assert not ck.exists()
    ref = g["prob_u16"].astype(np.float32) / np.float32(65535.0)
    e, e_own = np.abs(got - ref), np.abs(got - own)
    print(f"resumed the reference's checkpoint ({done}/{total} tiles done): vs reference max-abs {e.max():.3e}, "
          f"vs own uninterrupted run max-abs {e_own.max():.3e}")
    assert float(e.max()) <= 1e-2
    # the first tiles came from the reference's fp32 accumulator in the file, not from a rerun on the
    # GPU: they differ from the GPU's own f16 run by its rounding (a rerun would agree to ~1e-7)
    assert float(e_own.max()) > 1e-5
