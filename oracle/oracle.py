"""ctypes binding of the C oracle (oracle/fxo.c inference, oracle/fxv.c .fxvol codec) and a plain
Python reader of the .fxvol container. TEST INFRASTRUCTURE ONLY: imported by tests/,
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


class Spiral(C.Structure):
    _fields_ = [(k, C.c_double) for k in ("pitch", "thickness", "sheet_mean", "sheet_sd", "bg_mean", "bg_sd",
                                          "blur_sigma", "speckle_sd")]


# The synthetic volumes of the benchmark configurations (checker-side copy of the recipe).
SPIRAL_CONFIG1 = dict(pitch=12, thickness=3, sheet_mean=170, sheet_sd=15, bg_mean=40, bg_sd=10, blur_sigma=1.0,
                      speckle_sd=0.0)
SPIRAL_CONFIG3 = dict(SPIRAL_CONFIG1, pitch=16, speckle_sd=8.0)
SPIRAL_CONFIG5 = dict(SPIRAL_CONFIG1, pitch=14)


class Papyrus(C.Structure):
    _fields_ = [(k, C.c_double) for k in ("sigma_z", "sigma_y", "sigma_x", "mean", "sd", "ink_sigma", "ink_fraction",
                                          "ink_delta")]


# The layer-stack workload's papyrus with ink (checker-side copy of the recipe).
PAPYRUS_INK = dict(sigma_z=4.0, sigma_y=1.0, sigma_x=1.0, mean=110.0, sd=20.0, ink_sigma=6.0, ink_fraction=0.05,
                   ink_delta=25.0)


def synth_papyrus(shape, seed, stack=0, params=None, want_ink=False):
    """Papyrus layer stack [dz][dy][dx] u8 (+ its [dy][dx] ink mask) (oracle/synth.c)."""
    dz, dy, dx = shape
    p = Papyrus(**(params or PAPYRUS_INK))
    out = np.empty((dz, dy, dx), dtype=np.uint8)
    ink = np.empty((dy, dx), dtype=np.uint8)
    if lib().fxo_synth_papyrus(out.ctypes.data_as(C.POINTER(C.c_uint8)), ink.ctypes.data_as(C.POINTER(C.c_uint8)),
                               dz, dy, dx, C.byref(p), seed, stack):
        raise ValueError("fxo_synth_papyrus: bad arguments")
    return (out, ink) if want_ink else out


def synth_spiral(shape, seed, params=None, z_begin=0, z_end=None, chunked=False):
    """The spiral-sheet synthetic CT [z_end - z_begin][dy][dx] u8 (oracle/synth.c); chunked: noise
    keyed per 64^3 chunk."""
    dz, dy, dx = shape
    z_end = dz if z_end is None else z_end
    p = Spiral(**(params or SPIRAL_CONFIG1))
    out = np.empty((z_end - z_begin, dy, dx), dtype=np.uint8)
    fn = lib().fxo_synth_spiral_chunked if chunked else lib().fxo_synth_spiral
    if fn(out.ctypes.data_as(C.POINTER(C.c_uint8)), dz, dy, dx, C.byref(p), seed, z_begin, z_end):
        raise ValueError("fxo_synth_spiral: bad arguments")
    return out


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
        L.fxv_params_default.argtypes = [vp, C.c_float]
        L.fxv_dct3_fwd.argtypes = [f32p]
        L.fxv_dct3_inv.argtypes = [f32p]
        L.fxv_decode_tile.restype = i32
        L.fxv_decode_tile.argtypes = [vp, C.c_size_t, vp, f32p, u8p]
        L.fxv_encode_tile_u8.restype = i64
        L.fxv_encode_tile_u8.argtypes = [u8p, vp, i32, u8p, C.c_size_t]
        L.fxv_encode_tile_f32.restype = i64
        L.fxv_encode_tile_f32.argtypes = [f32p, vp, i32, u8p, C.c_size_t]
        L.fxv_log2_series.restype = C.c_double
        L.fxv_log2_series.argtypes = [C.c_double]
        L.fxv_crc32c.restype = C.c_uint32
        L.fxv_crc32c.argtypes = [vp, C.c_size_t]
        L.fxv_morton3.restype = C.c_uint64
        L.fxv_morton3.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64]
        L.fxo_synth_spiral.restype = i32
        L.fxo_synth_spiral.argtypes = [u8p, i64, i64, i64, C.POINTER(Spiral), C.c_uint64, i64, i64]
        L.fxo_synth_spiral_chunked.restype = i32
        L.fxo_synth_spiral_chunked.argtypes = [u8p, i64, i64, i64, C.POINTER(Spiral), C.c_uint64, i64, i64]
        L.fxo_net_forward_tiled.restype = i32
        L.fxo_net_forward_tiled.argtypes = [vp, f32p, i32, i32, i32, i32, i32, i32, f32p]
        L.fxo_predict_tiled.restype = i32
        L.fxo_predict_tiled.argtypes = [vp, u8p, i64, i64, i64, i32, i32, i32, C.c_double, i32, i32, f32p]
        L.fxo_synth_papyrus.restype = i32
        L.fxo_synth_papyrus.argtypes = [u8p, u8p, i64, i64, i64, C.POINTER(Papyrus), C.c_uint64, i64]
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

    def forward_tiled(self, x, channel=1, sigmoid=0):
        """x: [B][tz][ty][tx] normalised f32 -> selected-class probability, same shape."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros_like(x)
        if lib().fxo_net_forward_tiled(self.h, _fp(x), x.shape[0], *x.shape[1:], channel, sigmoid, _fp(out)):
            raise ValueError("oracle forward_tiled: the tile does not halve evenly through the stages")
        return out

    def predict_tiled(self, vol, tile, overlap, channel=1, sigmoid=0):
        """The sliding-window prediction with a (tz, ty, tx) tile (fxo_predict_tiled)."""
        v = np.ascontiguousarray(vol, dtype=np.uint8)
        out = np.zeros(v.shape, dtype=np.float32)
        if lib().fxo_predict_tiled(self.h, v.ctypes.data_as(C.POINTER(C.c_uint8)), *v.shape, *tile, overlap, channel,
                                   sigmoid, _fp(out)):
            raise ValueError("oracle predict_tiled failed")
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


def ref_infer(weights, vol, P, overlap, batch=1, threads=None, out_path=None, **opts):
    """Run the reference's own CPU predict_surface_filled (oracle/_ref/ref_infer). opts become its
    key=value options (tta, norm, channel, sigmoid, core=(z, y, x, dz, dy, dx), skipconst). Returns
    (prob, info dict); prob has the output's dims (the core's when cropped)."""
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
        for k, val in opts.items():
            cmd.append(f"{k}={','.join(map(str, val)) if isinstance(val, (tuple, list)) else val}")
        r = subprocess.run(cmd, capture_output=True, text=True, check=True)
        info = json.loads(r.stdout.strip().splitlines()[-1])
        prob = np.fromfile(op, dtype=np.float32).reshape(tuple(info.get("dims", v.shape)))
    return prob, info


# ---- .fxvol chunk codec (oracle/fxv.c) ----------------------------------------------------------

class FxvParams(C.Structure):
    """DctParams (src/codec/dct_block.hpp:26-37)."""

    _fields_ = [("q", C.c_float), ("hf_exp", C.c_float), ("dz_frac", C.c_float), ("rdoq", C.c_int),
                ("rdoq_lambda", C.c_float), ("deblock", C.c_int), ("deblock_beta", C.c_float),
                ("deblock_tc", C.c_float), ("dc_predict", C.c_int)]


def fxv_params(q: float, hf_exp: float = 0.65, dz_frac: float = 0.80) -> FxvParams:
    p = FxvParams()
    lib().fxv_params_default(C.byref(p), q)
    p.hf_exp, p.dz_frac = hf_exp, dz_frac
    return p


def fxv_decode(payload: bytes, q: float, hf_exp: float = 0.65, dz_frac: float = 0.80):
    """decode_tile_dct: (status, u8 tile, f32 reconstruction)."""
    b = np.frombuffer(payload, dtype=np.uint8) if payload else np.zeros(1, dtype=np.uint8)
    u8 = np.zeros((64, 64, 64), dtype=np.uint8)
    f = np.zeros((64, 64, 64), dtype=np.float32)
    p = fxv_params(q, hf_exp, dz_frac)
    rc = lib().fxv_decode_tile(b.ctypes.data, len(payload), C.byref(p), _fp(f), u8.ctypes.data_as(C.POINTER(C.c_uint8)))
    return rc, u8, f


def fxv_encode(tile: np.ndarray, q: float, log2_mode: int = 1, hf_exp: float = 0.65, dz_frac: float = 0.80) -> bytes:
    """encode_tile_dct of one 64^3 u8 or f32 tile; log2_mode 0 = glibc log2 (the reference's), 1 =
    the portable series (the device's)."""
    t = np.ascontiguousarray(tile)
    cap = 4 * 64 ** 3 + 4096
    out = np.zeros(cap, dtype=np.uint8)
    p = fxv_params(q, hf_exp, dz_frac)
    up = out.ctypes.data_as(C.POINTER(C.c_uint8))
    if t.dtype == np.uint8:
        n = lib().fxv_encode_tile_u8(t.ctypes.data_as(C.POINTER(C.c_uint8)), C.byref(p), log2_mode, up, cap)
    else:
        n = lib().fxv_encode_tile_f32(_fp(t.astype(np.float32, copy=False)), C.byref(p), log2_mode, up, cap)
    if n < 0:
        raise RuntimeError("fxv_encode failed")
    return out[:n].tobytes()


def fxv_dct3(block: np.ndarray, inverse: bool = False) -> np.ndarray:
    b = np.ascontiguousarray(block, dtype=np.float32).copy()
    (lib().fxv_dct3_inv if inverse else lib().fxv_dct3_fwd)(_fp(b))
    return b


def fxvol_read_slots(path) -> dict:
    """A plain reader of the .fxvol v5 container (src/codec/archive.hpp:42-130 layout, 161-262 open,
    1080-1107 radix walk): {"dims", "q", "hf_exp", "dz_frac", "nlods", "dtype", "slots"}, slots
    mapping (lod, cz, cy, cx) -> (coverage, payload or None) for every chunk of every LOD."""
    import struct

    buf = Path(path).read_bytes()
    best = None
    for s in range(2):
        b = buf[s * 4096:(s + 1) * 4096]
        magic, version = struct.unpack_from("<II", b, 0)
        crc_stored = struct.unpack_from("<I", b, 236)[0]
        if magic != 0x4C565846 or version != 5 or lib().fxv_crc32c(b, 236) != crc_stored:
            continue
        seq = struct.unpack_from("<Q", b, 8)[0]
        if best is None or seq > best[0]:
            best = (seq, b)
    if best is None:
        raise ValueError("no valid superblock")
    b = best[1]
    eof, nlods, dtype = struct.unpack_from("<QII", b, 16)
    dims = struct.unpack_from("<qqq", b, 32)
    q, hf, dzf = struct.unpack_from("<fff", b, 56)
    roots = struct.unpack_from("<20Q", b, 68)
    u64 = lambda off: struct.unpack_from("<Q", buf, off)[0]
    slots = {}
    d = list(dims)
    for lod in range(nlods):
        ce = [(v + 63) // 64 for v in d]
        for cz in range(ce[0]):
            for cy in range(ce[1]):
                for cx in range(ce[2]):
                    m = lib().fxv_morton3(cz, cy, cx)
                    cov, pay = 0, None
                    if roots[lod]:
                        c1 = u64(roots[lod] + 8 * ((m >> 24) & 0xFFF))
                        c2 = u64(c1 + 8 * ((m >> 12) & 0xFFF)) if c1 else 0
                        if c2:
                            off, n = struct.unpack_from("<QQ", buf, c2 + 16 * (m & 0xFFF))
                            if off != 0xFFFFFFFFFFFFFFFF:
                                cov = 1 if n == 0 else 2
                                if n:
                                    pay = buf[off:off + n]
                                    if struct.unpack_from("<I", buf, off + n)[0] != lib().fxv_crc32c(pay, n):
                                        raise ValueError("chunk crc mismatch")
                    slots[(lod, cz, cy, cx)] = (cov, pay)
        d = [(v + 1) // 2 for v in d]
    return {"dims": dims, "q": q, "hf_exp": hf, "dz_frac": dzf, "nlods": nlods, "dtype": dtype, "eof": eof,
            "slots": slots}


def fxvol_read_u8(path) -> np.ndarray:
    """read_volume_as<u8>(0) through the C oracle's tile decoder."""
    a = fxvol_read_slots(path)
    dz, dy, dx = a["dims"]
    out = np.zeros((dz, dy, dx), dtype=np.uint8)
    for (lod, cz, cy, cx), (cov, pay) in a["slots"].items():
        if lod or cov != 2:
            continue
        rc, t, _ = fxv_decode(pay, a["q"], a["hf_exp"], a["dz_frac"])
        if rc:
            raise ValueError(f"chunk {(cz, cy, cx)}: decode error {rc}")
        z0, y0, x0 = cz * 64, cy * 64, cx * 64
        sz, sy, sx = min(64, dz - z0), min(64, dy - y0), min(64, dx - x0)
        out[z0:z0 + sz, y0:y0 + sy, x0:x0 + sx] = t[:sz, :sy, :sx]
    return out
