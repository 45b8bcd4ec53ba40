"""A plain PyTorch fp32 model of the GPU path's arithmetic, used only as a test reference.

It computes the plain UNet with the same rounding points as the tensor-core path: conv / transposed
conv operands rounded to the layer's operand type (bf16, f16, or e4m3 with a per-tensor activation
scale and per-output-channel weight scales amax/448), f32 accumulation, the conv output stored
once as f16 before InstanceNorm (statistics from the unrounded f32 output), transposed-conv
output stored in the consumer's 16-bit type. With every type 'f32' it is the fp32 network the
reference computes.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

E4M3 = 448.0


def _round(t, kind, scale=None):
    if kind == "f32":
        return t
    if kind == "bf16":
        return t.to(torch.bfloat16).float()
    if kind == "f16":
        return t.clamp(-65504, 65504).to(torch.float16).float()
    if kind == "e4m3":
        return (t / scale).clamp(-E4M3, E4M3).to(torch.float8_e4m3fn).float() * scale
    raise ValueError(kind)


def _wq(w, kind, oc_dim):
    if kind != "e4m3":
        return _round(w, kind)
    dims = tuple(d for d in range(w.dim()) if d != oc_dim)
    s = w.abs().amax(dim=dims, keepdim=True).clamp(min=1e-8) / E4M3
    return (w / s).clamp(-E4M3, E4M3).to(torch.float8_e4m3fn).float() * s


def layer_keys(S, nconv=2):
    """Layer names in the library's order (fx_net_act_scales): encoder stage-major, transposed
    convs by output level (0 = finest), decoder convs level-major."""
    enc = [f"e{s}{i}" for s in range(S) for i in range(nconv)]
    up = [f"u{S - 2 - lvl}" for lvl in range(S - 1)]
    dec = [f"d{S - 2 - lvl}{i}" for lvl in range(S - 1) for i in range(nconv)]
    return enc + up + dec


def forward(params: dict, x: torch.Tensor, types: dict | None = None, scales: dict | None = None,
            default: str = "f32", prenorm: str | None = None, channel: int = 1) -> torch.Tensor:
    """x: [B,1,D,H,W] z-scored input. types/scales keyed by layer name (see layer_keys). A stage's
    stride is the kernel shape of the transposed conv that undoes it ((2, 2, 2), or (1, 2, 2) for a
    y/x-only stage); a one-class head is a sigmoid."""
    types = types or {}
    scales = scales or {}
    T = {k: torch.from_numpy(np.asarray(v)).to(x.device) for k, v in params.items()}
    S = sum(1 for k in T if k.startswith("encoder.stages.") and k.endswith(".convs.0.conv.weight"))
    nconv = sum(1 for k in T if k.startswith("encoder.stages.0.convs.") and k.endswith(".conv.weight"))
    pre_kind = prenorm if prenorm is not None else ("f32" if default == "f32" and not types else "f16")

    def ty(key):
        return types.get(key, default)

    def cna(x, pre, stride, key, act=True):
        k = ty(key)
        xi = _round(x, k, scales.get(key))
        wi = _wq(T[pre + ".conv.weight"], k, 0)
        y = F.conv3d(xi, wi, None, stride=stride, padding=1)
        m = y.mean(dim=(2, 3, 4), keepdim=True)
        v = y.var(dim=(2, 3, 4), unbiased=False, keepdim=True)
        y = _round(y, pre_kind)
        g = T[pre + ".norm.weight"].view(1, -1, 1, 1, 1)
        b = T[pre + ".norm.bias"].view(1, -1, 1, 1, 1)
        y = (y - m) / torch.sqrt(v + 1e-5) * g + b
        return F.leaky_relu(y, 0.01) if act else y

    stride = [(1, 1, 1)] + [tuple(T[f"decoder.transpconvs.{S - 1 - s}.weight"].shape[2:]) for s in range(1, S)]
    skips = []
    for s in range(S):
        for i in range(nconv):
            x = cna(x, f"encoder.stages.{s}.convs.{i}", stride[s] if i == 0 else 1, f"e{s}{i}")
        skips.append(x)
    for t in range(S - 1):
        lv = S - 2 - t
        key = f"u{t}"
        k = ty(key)
        up = F.conv_transpose3d(_round(x, k, scales.get(key)), _wq(T[f"decoder.transpconvs.{t}.weight"], k, 1),
                                T[f"decoder.transpconvs.{t}.bias"], stride=stride[lv + 1])
        x = torch.cat([up, skips[lv]], 1)
        for i in range(nconv):
            x = cna(x, f"decoder.stages.{t}.convs.{i}", 1, f"d{t}{i}")
    h = F.conv3d(x, T[f"decoder.seg_layers.{S - 2}.weight"], T[f"decoder.seg_layers.{S - 2}.bias"])
    if h.shape[1] == 1:
        return torch.sigmoid(h[:, 0])
    return torch.softmax(h, 1)[:, channel]


def gpu_types(features, precision: str, nconv: int = 2) -> dict:
    """Operand type of every layer in the library's nets: 16-bit layers are 'bf16' for bf16 nets
    and 'f16' otherwise; fp8 nets use e4m3 except the first conv and convs whose input channel
    count is not a multiple of 32. The first conv splits its operands into two 16-bit terms, which
    is modelled as fp32 operands."""
    S = len(features)
    t16 = "bf16" if precision == "bf16" else "f16"
    types = {}
    cin = {}
    prev = 1
    for s in range(S):
        for i in range(nconv):
            cin[f"e{s}{i}"] = prev if i == 0 else features[s]
        prev = features[s]
    for t in range(S - 1):
        lv = S - 2 - t
        cin[f"u{t}"] = features[lv + 1]
        for i in range(nconv):
            cin[f"d{t}{i}"] = 2 * features[lv] if i == 0 else features[lv]
    for k, c in cin.items():
        types[k] = "e4m3" if (precision == "fp8" and k != "e00" and c % 32 == 0) else t16
    types["e00"] = "f32"  # the first conv carries its input and weights as hi + lo 16-bit terms
    return types
