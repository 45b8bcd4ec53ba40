"""Octahedral test-time augmentation on the device (fx_infer_opts.tta) against its definition
(src/ml/infer.hpp:393-441): on a one-tile volume, the TTA prediction is the mean over members of
the plain prediction of the member-transformed volume, transformed back."""
import numpy as np
import pytest

import fenix_b200 as fx
from fenix_b200.weights import CONFIG1_FEATURES, make_plain_unet

pytestmark = pytest.mark.gpu

PERMS = [(0, 1, 2), (0, 2, 1), (1, 0, 2), (1, 2, 0), (2, 0, 1), (2, 1, 0)]


def forward_transform(v, m):
    pp, fm = PERMS[m // 8], m % 8
    x = np.transpose(v, pp)
    for d in range(3):
        if fm >> d & 1:
            x = np.flip(x, d)
    return np.ascontiguousarray(x)


def inverse_transform(p, m):
    pp, fm = PERMS[m // 8], m % 8
    for d in range(3):
        if fm >> d & 1:
            p = np.flip(p, d)
    q = [0, 0, 0]
    for d in range(3):
        q[pp[d]] = d
    return np.ascontiguousarray(np.transpose(p, q))


@pytest.mark.parametrize("tta", [8, 48])
def test_tta_is_member_mean(cuda_torch, tmp_path, tta):
    P = 64
    w = make_plain_unet(tmp_path / "c1.fxweights", CONFIG1_FEATURES, seed=0)
    vol = fx.synth_spiral((P, P, P), 21, fx.SPIRAL_CONFIG1)
    net = fx.Net(w, P, max_batch=8, precision="f16")
    got, _ = net.predict_volume(vol, overlap=0.5, batch=8, tta=tta)
    members = [inverse_transform(net.predict_volume(forward_transform(vol, m), overlap=0.5, batch=1)[0], m)
               for m in range(tta)]
    net.close()
    want = np.mean(np.stack(members), axis=0)
    assert np.abs(got - want).max() <= 2e-5
    # the members differ (the augmentation is not a no-op on this net)
    assert np.abs(members[0] - members[-1]).max() > 1e-3


def test_tta_one_is_plain(cuda_torch, tmp_path):
    P = 64
    w = make_plain_unet(tmp_path / "c1.fxweights", CONFIG1_FEATURES, seed=0)
    vol = fx.synth_spiral((96, 80, 72), 22, fx.SPIRAL_CONFIG1)
    net = fx.Net(w, P, max_batch=4, precision="f16")
    a, _ = net.predict_volume(vol, overlap=0.5, batch=4, tta=1)
    b, _ = net.predict_volume(vol, overlap=0.5, batch=4, tta=0)
    net.close()
    assert np.abs(a - b).max() <= 1e-6
