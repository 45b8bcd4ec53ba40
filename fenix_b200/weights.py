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

# Benchmark networks (features per stage)
CONFIG1_FEATURES = (16, 32, 64, 128)           # 4-stage, 2 classes
CONFIG2_FEATURES = (32, 64, 128, 256, 320)     # 5-stage nnU-Net style, 2 classes
# The layer-stack (wide-ink) net: 4 stages, 1 class + sigmoid, the first two strided stages halve y
# and x only (stride (1, 2, 2)), the last halves all three axes; 64 x 256 x 256 tiles
INK_FEATURES = (64, 128, 256, 512)
INK_STRIDES = ((1, 1, 1), (1, 2, 2), (1, 2, 2), (2, 2, 2))
INK_TILE = (64, 256, 256)


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


def plain_unet_params(features, nconv: int = 2, ncls: int = 2, seed: int = 0, strides=None) -> dict[str, np.ndarray]:
    """Seeded random init of the plain UNet. ``strides`` = per stage (z, y, x) stride of its first
    conv, each 1 or 2 (stage 0: (1, 1, 1)); None = 2 on every axis after stage 0. A stage's
    transposed conv has kernel = stride = that stage's stride, as nnU-Net builds it.

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
    if strides is None:
        strides = [(1, 1, 1)] + [(2, 2, 2)] * (S - 1)
    strides = [tuple(int(v) for v in st) for st in strides]
    if len(strides) != S or strides[0] != (1, 1, 1) or any(v not in (1, 2) for st in strides for v in st):
        raise ValueError("strides: one (z, y, x) triple of 1 / 2 per stage, stage 0 = (1, 1, 1)")
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
        # torch computes a ConvTranspose3d weight's fan_in from dim 1: Cout * prod(kernel)
        k = strides[S - 1 - t]
        P[f"decoder.transpconvs.{t}.weight"] = kaiming((below, skipc) + k, skipc * k[0] * k[1] * k[2])
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


def make_plain_unet(path: str | Path, features, nconv: int = 2, ncls: int = 2, seed: int = 0, strides=None) -> Path:
    write_fxweights(path, plain_unet_params(features, nconv, ncls, seed, strides))
    return Path(path)


def se_reduced(channels: int, rd_ratio: float = 1.0 / 16.0, divisor: int = 8) -> int:
    """The scSE bottleneck width: make_divisible(channels / 16, 8) (timm / nnU-Net)."""
    v = channels * rd_ratio
    return max(divisor, int(v + divisor / 2.0) // divisor * divisor)


def resenc_unet_params(features, blocks, ncls: int = 2, se: bool = False, plain_naming: bool = True,
                       task: str = "surface", seed: int = 0, task_head: bool = False) -> dict[str, np.ndarray]:
    """Seeded random init of the residual-encoder UNet (src/ml/nets/resenc_unet.hpp:55-318) with
    its checkpoint names: ``{enc}.stem.convs.0.*``, ``{enc}.stages.{s}.blocks.{b}.conv1/conv2.*``,
    ``...squeeze_excitation.cSE.fc1/fc2`` + ``sSE.conv`` (scSE), ``...skip.{i}.conv/norm`` (the 1x1
    projection after an optional AvgPool), and the plain decoder with one conv per stage.
    enc/dec = encoder/decoder (plain naming) or shared_encoder / task_decoders.<task>. Stage 0
    has stride 1, the others stride 2. Same draws as plain_unet_params."""
    import torch

    g = torch.Generator().manual_seed(int(seed))

    def kaiming(shape, fan_in):
        gain = (2.0 / (1 + 0.01 ** 2)) ** 0.5
        return (torch.randn(*shape, generator=g) * (gain / fan_in ** 0.5)).numpy()

    def small(n, base=0.0):
        return (base + 0.1 * torch.randn(n, generator=g)).numpy()

    if task_head:  # the ink checkpoints: shared_decoder without seg_layers + task_heads.<task>
        enc, dec = "shared_encoder", "shared_decoder"
    else:
        enc, dec = ("encoder", "decoder") if plain_naming else ("shared_encoder", f"task_decoders.{task}")
    P: dict[str, np.ndarray] = {}

    def cna(pre, cin, cout, k, bias=True):
        P[pre + ".conv.weight"] = kaiming((cout, cin, k, k, k), cin * k ** 3)
        if bias:
            P[pre + ".conv.bias"] = small(cout)
        P[pre + ".norm.weight"] = small(cout, 1.0)
        P[pre + ".norm.bias"] = small(cout)

    S = len(features)
    cna(f"{enc}.stem.convs.0", 1, features[0], 3)
    prev = features[0]
    for s in range(S):
        for b in range(blocks[s]):
            cin, cout = (prev if b == 0 else features[s]), features[s]
            stride = (1 if s == 0 else 2) if b == 0 else 1
            pre = f"{enc}.stages.{s}.blocks.{b}"
            cna(pre + ".conv1", cin, cout, 3)
            cna(pre + ".conv2", cout, cout, 3)
            if se:
                rd = se_reduced(cout)
                P[pre + ".squeeze_excitation.cSE.fc1.weight"] = kaiming((rd, cout, 1, 1, 1), cout)
                P[pre + ".squeeze_excitation.cSE.fc1.bias"] = small(rd)
                P[pre + ".squeeze_excitation.cSE.fc2.weight"] = kaiming((cout, rd, 1, 1, 1), rd)
                P[pre + ".squeeze_excitation.cSE.fc2.bias"] = small(cout)
                P[pre + ".squeeze_excitation.sSE.conv.weight"] = kaiming((1, cout, 1, 1, 1), cout)
                P[pre + ".squeeze_excitation.sSE.conv.bias"] = small(1)
            if cin != cout:  # projection; AvgPool (no parameters) takes index 0 when strided
                cna(pre + f".skip.{1 if stride != 1 else 0}", cin, cout, 1, bias=False)
        prev = features[s]
    for t in range(S - 1):
        below, skipc = features[S - 1 - t], features[S - 2 - t]
        P[f"{dec}.transpconvs.{t}.weight"] = kaiming((below, skipc, 2, 2, 2), skipc * 8)
        P[f"{dec}.transpconvs.{t}.bias"] = small(skipc)
        cna(f"{dec}.stages.{t}.convs.0", 2 * skipc, skipc, 3)
        if not task_head:
            P[f"{dec}.seg_layers.{t}.weight"] = kaiming((ncls, skipc, 1, 1, 1), skipc)
            P[f"{dec}.seg_layers.{t}.bias"] = small(ncls)
    if task_head:
        P[f"task_heads.{task}.weight"] = kaiming((ncls, features[0], 1, 1, 1), features[0])
        P[f"task_heads.{task}.bias"] = small(ncls)
    return P


def make_resenc_unet(path: str | Path, features, blocks, ncls: int = 2, se: bool = False,
                     plain_naming: bool = True, seed: int = 0, task: str = "surface", task_head: bool = False) -> Path:
    write_fxweights(path, resenc_unet_params(features, blocks, ncls, se, plain_naming, task, seed, task_head))
    return Path(path)
