"""Seeded random-init plain UNets written as .fxweights, on the checker side. TEST INFRASTRUCTURE
ONLY: the benchmark's reference arm and the fixture scripts make the workload's network with it
without importing the product package; a CPU test checks that its files equal the product's
(fenix_b200.weights.make_plain_unet) byte for byte.

Format: the reference's FXWT v1 (src/ml/weights.hpp:1-10): "FXWT" | u32 version 1 | u32 count |
u32 reserved, then per tensor u16 name length | name | u8 dtype (0 = f32) | u8 ndim | u64 bytes |
u64 data offset | i64 shape[ndim], blobs 64-byte aligned. Names follow the reference's plain
nnU-Net module naming (src/ml/nets/resenc_unet.hpp:141-239). Draws: torch's CPU generator seeded
with `seed`, in module order; conv / transposed-conv weights Kaiming-normal (leaky_relu gain with
a = 1e-2, fan_in), biases 0.1 N(0,1), InstanceNorm weight 1 + 0.1 N(0,1), bias 0.1 N(0,1).
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np


def plain_unet(features, nconv=2, ncls=2, seed=0, strides=None):
    """strides: per stage (z, y, x) stride of its first conv (stage 0 (1, 1, 1)); None = 2 on every
    axis after stage 0. The transposed conv undoing a stage has kernel = stride (nnU-Net's
    get_network_from_plans: transpconv_op(..., pool_op_kernel_sizes[s], stride=pool_op_kernel_sizes[s]))."""
    import torch

    g = torch.Generator().manual_seed(int(seed))
    gain = (2.0 / (1 + 0.01 ** 2)) ** 0.5
    out = {}

    def normal(shape, sd, base=0.0):
        return (base + sd * torch.randn(*shape, generator=g)).numpy()

    S = len(features)
    strides = [(1, 1, 1)] + [(2, 2, 2)] * (S - 1) if strides is None else [tuple(st) for st in strides]
    cin = 1
    for s in range(S):
        for i in range(nconv):
            c_in = cin if i == 0 else features[s]
            pre = f"encoder.stages.{s}.convs.{i}"
            out[pre + ".conv.weight"] = normal((features[s], c_in, 3, 3, 3), gain / (c_in * 27) ** 0.5)
            out[pre + ".conv.bias"] = normal((features[s],), 0.1)
            out[pre + ".norm.weight"] = normal((features[s],), 0.1, 1.0)
            out[pre + ".norm.bias"] = normal((features[s],), 0.1)
        cin = features[s]
    for t in range(S - 1):
        below, skipc = features[S - 1 - t], features[S - 2 - t]
        k = strides[S - 1 - t]
        out[f"decoder.transpconvs.{t}.weight"] = normal((below, skipc) + k, gain / (skipc * k[0] * k[1] * k[2]) ** 0.5)
        out[f"decoder.transpconvs.{t}.bias"] = normal((skipc,), 0.1)
        for i in range(nconv):
            c_in = 2 * skipc if i == 0 else skipc
            pre = f"decoder.stages.{t}.convs.{i}"
            out[pre + ".conv.weight"] = normal((skipc, c_in, 3, 3, 3), gain / (c_in * 27) ** 0.5)
            out[pre + ".conv.bias"] = normal((skipc,), 0.1)
            out[pre + ".norm.weight"] = normal((skipc,), 0.1, 1.0)
            out[pre + ".norm.bias"] = normal((skipc,), 0.1)
        out[f"decoder.seg_layers.{t}.weight"] = normal((ncls, skipc, 1, 1, 1), gain / skipc ** 0.5)
        out[f"decoder.seg_layers.{t}.bias"] = normal((ncls,), 0.1)
    return out


def write_fxweights(path, tensors):
    items = [(k.encode(), np.ascontiguousarray(v, dtype=np.float32)) for k, v in tensors.items()]
    head = b"FXWT" + struct.pack("<III", 1, len(items), 0)
    table_len = sum(2 + len(n) + 2 + 16 + 8 * a.ndim for n, a in items)
    off = (len(head) + table_len + 63) // 64 * 64
    table, offs = bytearray(), []
    for n, a in items:
        offs.append(off)
        table += struct.pack("<H", len(n)) + n + struct.pack("<BBQQ", 0, a.ndim, a.nbytes, off)
        table += struct.pack(f"<{a.ndim}q", *a.shape)
        off = (off + a.nbytes + 63) // 64 * 64
    buf = bytearray(off)
    buf[:len(head) + len(table)] = head + table
    for (n, a), o in zip(items, offs):
        buf[o:o + a.nbytes] = a.tobytes()
    Path(path).write_bytes(bytes(buf))
    return Path(path)


def make_plain_unet(path, features, nconv=2, ncls=2, seed=0, strides=None):
    return write_fxweights(path, plain_unet(features, nconv, ncls, seed, strides))
