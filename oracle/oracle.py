"""ctypes binding of the C oracle (oracle/fxo.c). TEST INFRASTRUCTURE ONLY: imported by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg as the checker; the product never
imports it."""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"
REF = HERE / "_ref"
_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = C.CDLL(str(LIB))
        i64, i32, f32p, u8p, vp = C.c_int64, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_uint8), C.c_void_p
        L.fxo_tile_starts.restype = i64
        L.fxo_tile_starts.argtypes = [i64, i32, C.c_double, C.POINTER(C.c_int64), i64]
        L.fxo_gaussian1d.argtypes = [i32, f32p]
        L.fxo_weight_profile.argtypes = [f32p, i32, C.POINTER(C.c_int64), i64, i64, i64, i64, f32p]
        L.fxo_fill_patch_u8.argtypes = [u8p, i64, i64, i64, i64, i64, i64, i32, f32p]
        L.fxo_norm_patch_zscore.argtypes = [f32p, i32]
        L.fxo_net_load.restype = vp
        L.fxo_net_load.argtypes = [C.c_char_p]
        L.fxo_net_free.argtypes = [vp]
        L.fxo_net_forward.argtypes = [vp, f32p, i32, i32, i32, i32, f32p]
        L.fxo_predict_surface.argtypes = [vp, u8p, i64, i64, i64, i32, C.c_double, i32, i32, f32p]
        L.fxo_prob_to_u8.argtypes = [f32p, i64, u8p]
        _lib = L
    return _lib


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def tile_starts(dim, patch, overlap):
    n = lib().fxo_tile_starts(dim, patch, overlap, None, 0)
    out = np.zeros(n, dtype=np.int64)
    lib().fxo_tile_starts(dim, patch, overlap, out.ctypes.data_as(C.POINTER(C.c_int64)), n)
    return out


def gaussian1d(n):
    out = np.zeros(n, dtype=np.float32)
    lib().fxo_gaussian1d(n, _fp(out))
    return out


def weight_profile(g, patch, starts, c0, cn, dim):
    g = np.ascontiguousarray(g, dtype=np.float32)
    st = np.ascontiguousarray(starts, dtype=np.int64)
    out = np.zeros(cn, dtype=np.float32)
    lib().fxo_weight_profile(_fp(g), patch, st.ctypes.data_as(C.POINTER(C.c_int64)), len(st), c0, cn, dim, _fp(out))
    return out


def norm_tile(vol, origin, P):
    """Fill (edge clamp) + z-score one tile, f32 [P^3]."""
    v = np.ascontiguousarray(vol, dtype=np.uint8)
    out = np.zeros((P, P, P), dtype=np.float32)
    lib().fxo_fill_patch_u8(v.ctypes.data_as(C.POINTER(C.c_uint8)), *v.shape, *origin, P, _fp(out))
    lib().fxo_norm_patch_zscore(_fp(out), P)
    return out


class Net:
    def __init__(self, path):
        self.h = lib().fxo_net_load(str(path).encode())
        if not self.h:
            raise ValueError(f"oracle: cannot load {path}")

    def __del__(self):
        if getattr(self, "h", None):
            lib().fxo_net_free(self.h)

    def forward(self, x, channel=1, sigmoid=0):
        """x: [B][P][P][P] normalised f32 -> selected-class probability, same shape."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        B, P = x.shape[0], x.shape[1]
        out = np.zeros_like(x)
        lib().fxo_net_forward(self.h, _fp(x), B, P, channel, sigmoid, _fp(out))
        return out

    def predict_surface(self, vol, P, overlap, channel=1, sigmoid=0):
        v = np.ascontiguousarray(vol, dtype=np.uint8)
        out = np.zeros(v.shape, dtype=np.float32)
        rc = lib().fxo_predict_surface(self.h, v.ctypes.data_as(C.POINTER(C.c_uint8)), *v.shape, P, overlap, channel,
                                       sigmoid, _fp(out))
        if rc != 0:
            raise ValueError("oracle predict_surface failed")
        return out


def prob_to_u8(p):
    p = np.ascontiguousarray(p, dtype=np.float32)
    out = np.zeros(p.shape, dtype=np.uint8)
    lib().fxo_prob_to_u8(_fp(p), p.size, out.ctypes.data_as(C.POINTER(C.c_uint8)))
    return out


def ref_infer(weights, vol, P, overlap, batch=1, threads=None, out_path=None):
    """Run the reference's own CPU predict_surface_filled (oracle/_ref/ref_infer). Returns
    (prob or None, info dict)."""
    import json
    import tempfile

    exe = REF / "ref_infer"
    if not exe.exists():
        raise FileNotFoundError(exe)
    v = np.ascontiguousarray(vol, dtype=np.uint8)
    with tempfile.TemporaryDirectory() as td:
        vp = Path(td) / "vol.u8"
        v.tofile(vp)
        op = Path(td) / "prob.f32" if out_path is None else Path(out_path)
        cmd = [str(exe), str(weights), str(vp), *map(str, v.shape), str(P), str(overlap), str(batch), str(op)]
        if threads:
            cmd.append(str(threads))
        r = subprocess.run(cmd, capture_output=True, text=True, check=True)
        info = json.loads(r.stdout.strip().splitlines()[-1])
        prob = np.fromfile(op, dtype=np.float32).reshape(v.shape)
    return prob, info
