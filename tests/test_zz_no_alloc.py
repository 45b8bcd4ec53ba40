"""fx_norm_tiles_noalloc: the tile z-score over a static device scratch, against fx_norm_tiles.

The file sorts last so that the static scratch is first used after every other test has run on
the device, and the same checks hold when the file runs alone.
"""
import ctypes as C

import numpy as np
import pytest

import fenix_b200 as fx

MAX_TILES = 4096  # the static scratch's capacity per call
FX_INVALID_ARGUMENT = 1


def _org_ptr(a):
    return a.ctypes.data_as(C.POINTER(C.c_int64))


def _norm(fn, dv, shape, org, P, out):
    fx.check(getattr(fx.lib(), fn)(dv.data_ptr(), *shape, _org_ptr(org), len(org), P, out.data_ptr(), None))


@pytest.mark.gpu
def test_noalloc_matches_norm_tiles_two_calls(cuda_torch):
    torch = cuda_torch
    vol = fx.synth_spiral((70, 50, 90), 9)
    dv = torch.from_numpy(vol).cuda()
    P = 32
    # the last origin of the first set runs past all three edges (edge-clamped reads); the second
    # set repeats two tiles, so sums left over from the first call would change its result
    sets = [np.array([[0, 0, 0], [6, 0, 26], [38, 18, 58], [50, 30, 70]], dtype=np.int64),
            np.array([[10, 4, 2], [0, 0, 0], [38, 18, 58]], dtype=np.int64)]
    got = []
    for org in sets:  # two calls in a row
        out = torch.full((len(org), P, P, P), float("nan"), device="cuda")
        _norm("fx_norm_tiles_noalloc", dv, vol.shape, org, P, out)
        got.append(out)
    for org, g in zip(sets, got):
        want = torch.zeros((len(org), P, P, P), device="cuda")
        _norm("fx_norm_tiles", dv, vol.shape, org, P, want)
        torch.cuda.synchronize()
        assert torch.equal(g, want)  # the z-score is bit-exact: tolerance 0


@pytest.mark.gpu
def test_noalloc_at_capacity_and_beyond(cuda_torch):
    torch = cuda_torch
    vol = fx.synth_spiral((40, 36, 44), 5)
    dv = torch.from_numpy(vol).cuda()
    P = 4
    rng = np.random.default_rng(7)
    org = np.stack([rng.integers(0, d - P + 3, MAX_TILES) for d in vol.shape], axis=1).astype(np.int64)
    for _ in range(2):
        got = torch.full((MAX_TILES, P, P, P), float("nan"), device="cuda")
        _norm("fx_norm_tiles_noalloc", dv, vol.shape, org, P, got)
        want = torch.zeros_like(got)
        _norm("fx_norm_tiles", dv, vol.shape, org, P, want)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    over = np.zeros((MAX_TILES + 1, 3), dtype=np.int64)
    big = torch.zeros((MAX_TILES + 1, P, P, P), device="cuda")
    st = fx.lib().fx_norm_tiles_noalloc(dv.data_ptr(), *vol.shape, _org_ptr(over), MAX_TILES + 1, P,
                                        big.data_ptr(), None)
    assert st == FX_INVALID_ARGUMENT
    assert b"static scratch limit of 4096" in fx.lib().fx_last_error()
    assert not big.any()


def test_noalloc_rejects_oversize_before_device_work():
    """The size check comes before any CUDA call, so it answers on a machine without a GPU."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("covered with device buffers by test_noalloc_at_capacity_and_beyond")
    over = np.zeros((MAX_TILES + 1, 3), dtype=np.int64)
    host = np.zeros(16, dtype=np.uint8)
    st = fx.lib().fx_norm_tiles_noalloc(host.ctypes.data, 8, 8, 8, _org_ptr(over), MAX_TILES + 1, 4,
                                        host.ctypes.data, None)
    assert st == FX_INVALID_ARGUMENT
    assert b"static scratch limit" in fx.lib().fx_last_error()
