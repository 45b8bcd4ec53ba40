"""Parity of the tcgen05 conv kernel (through the C ABI) against a plain PyTorch fp32 reference.

The operands the kernel sees are rounded (bf16, f16, or e4m3 with per-output-channel weight
scales and a per-tensor input scale), so the reference convolves the same rounded operands in
fp32; the kernel accumulates in fp32 and stores its output once as f16, so the tolerance is
2^-7 relative plus 2e-3 of the output's scale (rounding of the f16 store and fp32
summation-order noise).
"""
import ctypes as C

import numpy as np
import pytest

import fenix_b200 as fx

pytestmark = pytest.mark.gpu

E4M3 = 448.0


PREC = {"bf16": 0, "fp8": 1, "f16": 2}


def _q16(t, kind):
    import torch

    return t.to(torch.bfloat16 if kind == "bf16" else torch.float16).float()


def _q_e4m3_tensor(t):
    import torch

    s = t.abs().max().clamp(min=1e-8) / E4M3
    return (t / s).to(torch.float8_e4m3fn).float() * s


def _q_e4m3_per_oc(w):
    import torch

    dims = tuple(range(1, w.dim()))
    s = w.abs().amax(dim=dims, keepdim=True).clamp(min=1e-8) / E4M3
    return (w / s).to(torch.float8_e4m3fn).float() * s


def _close(y, ref, rel=2.0 ** -7, abs_frac=2e-3):
    scale = ref.abs().max().item()
    err = (y - ref).abs()
    bound = rel * ref.abs() + abs_frac * scale
    bad = (err > bound).sum().item()
    return bad, err.max().item(), scale


CONV_CASES = [
    # B, Cin, Cout, (D, H, W), stride
    (1, 16, 32, (8, 8, 8), 1),
    (1, 16, 16, (8, 8, 8), 1),
    (2, 32, 32, (12, 10, 20), 1),
    (1, 64, 64, (16, 16, 16), 1),
    (1, 32, 64, (16, 16, 16), 2),
    (2, 64, 128, (8, 12, 8), 2),
    (1, 128, 256, (8, 8, 8), 1),
    (1, 256, 320, (4, 4, 4), 2),
    (1, 320, 320, (4, 4, 4), 1),
    (1, 1, 32, (16, 12, 20), 1),  # the 1-channel first layer (x-folded taps, hi + lo split)
    (1, 32, 32, (3, 5, 7), 1),     # fewer rows than one M block
    (2, 32, 16, (20, 14, 30), 1),
    (1, 64, 32, (24, 20, 18), 1),
]


def _foldable(Cin, Cout, stride):
    return stride == 1 and Cin > 1 and Cout in (16, 32, 64)


@pytest.fixture(params=["fold", "nofold"])
def fold_mode(request, monkeypatch):
    """Stride-1 convs with 16/32/64 output channels run the x-tap fold when
    FENIX_B200_CONV_FOLD=1: test both programs."""
    monkeypatch.setenv("FENIX_B200_CONV_FOLD", "1" if request.param == "fold" else "0")
    return request.param


@pytest.mark.parametrize("kind", ["bf16", "f16"])
@pytest.mark.parametrize("B,Cin,Cout,dims,stride", CONV_CASES)
def test_conv3d_16bit(cuda_torch, fold_mode, B, Cin, Cout, dims, stride, kind):
    torch = cuda_torch
    import torch.nn.functional as F

    if fold_mode == "nofold" and not _foldable(Cin, Cout, stride):
        pytest.skip("same program either way")

    g = torch.Generator().manual_seed(1000 + Cin * 7 + Cout + stride)
    D, H, W = dims
    x = torch.randn(B, Cin, D, H, W, generator=g)
    w = torch.randn(Cout, Cin, 3, 3, 3, generator=g) * (2.0 / (27 * Cin)) ** 0.5
    # the 1-channel first layer carries input and weights as hi + lo 16-bit terms (about fp32)
    xq, wq = (x, w) if Cin == 1 else (_q16(x, kind), _q16(w, kind))
    ref = F.conv3d(xq, wq, stride=stride, padding=1)
    xd, wd = x.cuda(), w.cuda()
    y = torch.zeros_like(ref, device="cuda")
    st = torch.zeros(B, Cout, 2, device="cuda")
    fx.check(fx.lib().fx_conv3d(xd.data_ptr(), B, Cin, D, H, W, wd.data_ptr(), Cout, stride, PREC[kind],
                                y.data_ptr(), st.data_ptr(), None))
    torch.cuda.synchronize()
    bad, emax, scale = _close(y.cpu(), ref)
    assert bad == 0, f"{bad} mismatches, max err {emax} (ref scale {scale})"
    mean = ref.mean(dim=(2, 3, 4))
    var = ref.var(dim=(2, 3, 4), unbiased=False)
    stc = st.cpu()
    assert torch.allclose(stc[..., 0], mean, atol=1e-4 * scale, rtol=1e-4)
    assert torch.allclose(stc[..., 1], var, atol=1e-4 * scale * scale, rtol=1e-3)


@pytest.mark.parametrize("B,Cin,Cout,dims,stride", [c for c in CONV_CASES if c[1] >= 32])
def test_conv3d_fp8(cuda_torch, fold_mode, B, Cin, Cout, dims, stride):
    torch = cuda_torch
    import torch.nn.functional as F

    if fold_mode == "nofold" and not _foldable(Cin, Cout, stride):
        pytest.skip("same program either way")

    g = torch.Generator().manual_seed(2000 + Cin * 7 + Cout + stride)
    D, H, W = dims
    x = torch.randn(B, Cin, D, H, W, generator=g)
    w = torch.randn(Cout, Cin, 3, 3, 3, generator=g) * (2.0 / (27 * Cin)) ** 0.5
    ref = F.conv3d(_q_e4m3_tensor(x), _q_e4m3_per_oc(w), stride=stride, padding=1)
    xd, wd = x.cuda(), w.cuda()
    y = torch.zeros_like(ref, device="cuda")
    fx.check(fx.lib().fx_conv3d(xd.data_ptr(), B, Cin, D, H, W, wd.data_ptr(), Cout, stride, 1, y.data_ptr(), None,
                                None))
    torch.cuda.synchronize()
    bad, emax, scale = _close(y.cpu(), ref)
    assert bad == 0, f"{bad} mismatches, max err {emax} (ref scale {scale})"


UP_CASES = [
    (1, 64, 32, (8, 8, 8)),
    (2, 32, 16, (6, 10, 8)),
    (1, 128, 64, (8, 8, 8)),
    (1, 256, 128, (4, 6, 4)),
    (1, 320, 256, (4, 4, 4)),
]


@pytest.mark.parametrize("kind", ["bf16", "f16", "fp8"])
@pytest.mark.parametrize("B,Cin,Cout,dims", UP_CASES)
def test_conv_transpose2(cuda_torch, B, Cin, Cout, dims, kind):
    torch = cuda_torch
    import torch.nn.functional as F

    fp8 = kind == "fp8"
    if fp8 and (Cin % 32 or Cout % 16):
        pytest.skip("fp8 needs Cin % 32 == 0 and Cout % 16 == 0")
    g = torch.Generator().manual_seed(3000 + Cin + Cout)
    D, H, W = dims
    x = torch.randn(B, Cin, D, H, W, generator=g)
    w = torch.randn(Cin, Cout, 2, 2, 2, generator=g) * (1.0 / (8 * Cout)) ** 0.5
    b = torch.randn(Cout, generator=g) * 0.1
    if fp8:
        xq = _q_e4m3_tensor(x)
        s = w.abs().amax(dim=(0, 2, 3, 4), keepdim=True).clamp(min=1e-8) / E4M3
        wq = (w / s).to(torch.float8_e4m3fn).float() * s
    else:
        xq, wq = _q16(x, kind), _q16(w, kind)
    ref = F.conv_transpose3d(xq, wq, b, stride=2)
    y = torch.zeros_like(ref, device="cuda")
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    fx.check(fx.lib().fx_conv_transpose2(xd.data_ptr(), B, Cin, D, H, W, wd.data_ptr(), bd.data_ptr(), Cout,
                                         PREC[kind], y.data_ptr(), None))
    torch.cuda.synchronize()
    bad, emax, scale = _close(y.cpu(), ref)
    assert bad == 0, f"{bad} mismatches, max err {emax} (ref scale {scale})"
