"""`.fxweights` (FXWT v1) writer and the seeded random-init plain UNet used by tests and the benchmark.

File layout (little-endian), the reference's flat tensor format (src/ml/weights.hpp:1-10):
``"FXWT" | u32 version=1 | u32 count | u32 reserved`` then per tensor
``u16 name_len | name | u8 dtype | u8 ndim | u64 nbytes | u64 data_off | i64 shape[ndim]``,
blobs 64-byte aligned. Only dtype 0 (f32) is written.

Parameter names follow the reference's module naming for a plain nnU-Net UNet composed of its
``ConvStack`` / ``ConvTranspose3d`` / ``Conv3d`` modules (src/ml/nets/resenc_unet.hpp:141-239):
``encoder.stages.{s}.convs.{i}.conv.{weight,bias}``, ``...norm.{weight,bias}``,
``decoder.transpconvs.{t}.{weight,bias}``, ``decoder.stages.{t}.convs.{i}.*`` and
``decoder.seg_layers.{t}.{weight,bias}`` (t = 0 is the deepest decoder stage).
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

# BASELINE networks (features per stage)
CONFIG1_FEATURES = (16, 32, 64, 128)           # 4-stage, 2 classes
CONFIG2_FEATURES = (32, 64, 128, 256, 320)     # 5-stage nnU-Net style, 2 classes


def write_fxweights(path: str | Path, tensors: dict[str, np.ndarray]) -> None:
    items = [(k, np.ascontiguousarray(v, dtype=np.float32)) for k, v in tensors.items()]
    header = bytearray(b"FXWT" + struct.pack("<III", 1, len(items), 0))
    recs = []
    for name, arr in items:
        nb = name.encode()
        recs.append((nb, arr))
    # compute record table size to place blobs after it
    table = 0
    for nb, arr in recs:
        table += 2 + len(nb) + 1 + 1 + 8 + 8 + 8 * arr.ndim
    off = len(header) + table
    off = (off + 63) // 64 * 64
    offsets = []
    for nb, arr in recs:
        offsets.append(off)
        off = (off + arr.nbytes + 63) // 64 * 64
    out = bytearray(header)
    for (nb, arr), o in zip(recs, offsets):
        out += struct.pack("<H", len(nb)) + nb + struct.pack("<BB", 0, arr.ndim)
        out += struct.pack("<QQ", arr.nbytes, o)
        out += struct.pack(f"<{arr.ndim}q", *arr.shape)
    blob = bytearray(off)
    blob[: len(out)] = out
    for (nb, arr), o in zip(recs, offsets):
        blob[o : o + arr.nbytes] = arr.tobytes()
    Path(path).write_bytes(bytes(blob))


def read_fxweights(path: str | Path) -> dict[str, np.ndarray]:
    b = Path(path).read_bytes()
    assert b[:4] == b"FXWT"
    ver, cnt, _ = struct.unpack_from("<III", b, 4)
    assert ver == 1
    cur = 16
    out = {}
    for _ in range(cnt):
        (nl,) = struct.unpack_from("<H", b, cur)
        cur += 2
        name = b[cur : cur + nl].decode()
        cur += nl
        dt, nd = struct.unpack_from("<BB", b, cur)
        cur += 2
        nbytes, off = struct.unpack_from("<QQ", b, cur)
        cur += 16
        shape = struct.unpack_from(f"<{nd}q", b, cur)
        cur += 8 * nd
        assert dt == 0
        out[name] = np.frombuffer(b, dtype=np.float32, count=nbytes // 4, offset=off).reshape(shape).copy()
    return out


def plain_unet_params(features, nconv: int = 2, ncls: int = 2, seed: int = 0) -> dict[str, np.ndarray]:
    """Seeded random init of the plain UNet.

    Conv and transposed-conv weights are Kaiming-normal (torch.nn.init.kaiming_normal_ with
    a=1e-2, fan_in, leaky_relu gain, the nnU-Net convention) drawn from torch's CPU generator
    seeded with ``seed``, in module order. Biases and the InstanceNorm affine parameters are
    drawn small and non-trivial (not the usual 0 / 1) so that every bias and affine path of
    the kernels is exercised: conv/transposed-conv/head biases ~ 0.1 N(0,1), InstanceNorm
    weight ~ 1 + 0.1 N(0,1), InstanceNorm bias ~ 0.1 N(0,1).
    """
    import torch

    g = torch.Generator().manual_seed(int(seed))

    def kaiming(shape, fan_in):
        gain = (2.0 / (1 + 0.01 ** 2)) ** 0.5
        return (torch.randn(*shape, generator=g) * (gain / fan_in ** 0.5)).numpy()

    def small(n, base=0.0):
        return (base + 0.1 * torch.randn(n, generator=g)).numpy()

    P: dict[str, np.ndarray] = {}
    S = len(features)
    prev = 1
    for s in range(S):
        for i in range(nconv):
            cin = prev if i == 0 else features[s]
            cout = features[s]
            pre = f"encoder.stages.{s}.convs.{i}"
            P[pre + ".conv.weight"] = kaiming((cout, cin, 3, 3, 3), cin * 27)
            P[pre + ".conv.bias"] = small(cout)
            P[pre + ".norm.weight"] = small(cout, 1.0)
            P[pre + ".norm.bias"] = small(cout)
        prev = features[s]
    for t in range(S - 1):
        below, skipc = features[S - 1 - t], features[S - 2 - t]
        # torch computes a ConvTranspose3d weight's fan_in from dim 1: Cout * 8
        P[f"decoder.transpconvs.{t}.weight"] = kaiming((below, skipc, 2, 2, 2), skipc * 8)
        P[f"decoder.transpconvs.{t}.bias"] = small(skipc)
        for i in range(nconv):
            cin = 2 * skipc if i == 0 else skipc
            pre = f"decoder.stages.{t}.convs.{i}"
            P[pre + ".conv.weight"] = kaiming((skipc, cin, 3, 3, 3), cin * 27)
            P[pre + ".conv.bias"] = small(skipc)
            P[pre + ".norm.weight"] = small(skipc, 1.0)
            P[pre + ".norm.bias"] = small(skipc)
        P[f"decoder.seg_layers.{t}.weight"] = kaiming((ncls, skipc, 1, 1, 1), skipc)
        P[f"decoder.seg_layers.{t}.bias"] = small(ncls)
    return P


def make_plain_unet(path: str | Path, features, nconv: int = 2, ncls: int = 2, seed: int = 0) -> Path:
    write_fxweights(path, plain_unet_params(features, nconv, ncls, seed))
    return Path(path)
