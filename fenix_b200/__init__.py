"""fenix_b200 — B200 (sm_100a) surface-prediction inference: Python bindings over the C ABI.

Every call goes through ``libfenix_b200.so`` (the ``extern "C"`` functions declared in
``include/fenix_b200.h``). There is no Python or CPU fallback for any compute entry point: when
the library is missing, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "_build" / "libfenix_b200.so"
_lib = None

FX_OK = 0
FX_INVALID_ARGUMENT = 1
STATUS_NAMES = {
    0: "ok",
    1: "invalid_argument",
    2: "not_found",
    3: "io_error",
    4: "fetch_failed",
    5: "decode_error",
    6: "unsupported",
    7: "unimplemented",
    8: "internal",
}
PREC_BF16, PREC_FP8, PREC_F16 = 0, 1, 2
PRECISIONS = {"bf16": PREC_BF16, "fp8": PREC_FP8, "f16": PREC_F16}


class FxError(RuntimeError):
    """A non-zero fx_status from the library; ``code`` holds the status, the message fx_last_error()."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


TileFilter = C.CFUNCTYPE(C.c_int, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_void_p)
NORMS = {"zscore": 0, "pct_minmax": 1, "unit255": 2}


class InferOpts(C.Structure):
    """fx_infer_opts (mirrors the reference's ml::InferOptions): fields after tta default to zero =
    zscore, every tile, no crop, no filter."""

    _fields_ = [
        ("patch", C.c_int),
        ("overlap", C.c_double),
        ("channel", C.c_int),
        ("sigmoid", C.c_int),
        ("batch", C.c_int),
        ("tta", C.c_int),
        ("norm", C.c_int),
        ("skip_constant", C.c_int),
        ("core_org", C.c_int64 * 3),
        ("core_ext", C.c_int64 * 3),
        ("tile_filter", TileFilter),
        ("tile_filter_user", C.c_void_p),
        ("tile", C.c_int * 3),
        ("stacks", C.c_int),
        ("ckpt_path", C.c_char_p),
        ("ckpt_every", C.c_int64),
        ("weights_hash", C.c_uint64),
        ("input_hash", C.c_uint64),
    ]


class PapyrusParams(C.Structure):
    """fx_papyrus_params (include/fenix_b200_synth.h)."""

    _fields_ = [(k, C.c_double) for k in ("sigma_z", "sigma_y", "sigma_x", "mean", "sd", "ink_sigma", "ink_fraction",
                                          "ink_delta")]


# The layer-stack workload's papyrus: fibre texture sigma (4, 1, 1) around 110 +- 20, ink blobs
# (2D sigma 6) on 5% of the (y, x) columns, +25.
PAPYRUS_INK = dict(sigma_z=4.0, sigma_y=1.0, sigma_x=1.0, mean=110.0, sd=20.0, ink_sigma=6.0, ink_fraction=0.05,
                   ink_delta=25.0)


class SpiralParams(C.Structure):
    """fx_spiral_params (include/fenix_b200_synth.h)."""

    _fields_ = [
        ("pitch", C.c_double),
        ("thickness", C.c_double),
        ("sheet_mean", C.c_double),
        ("sheet_sd", C.c_double),
        ("bg_mean", C.c_double),
        ("bg_sd", C.c_double),
        ("blur_sigma", C.c_double),
        ("speckle_sd", C.c_double),
    ]


# Synthetic volumes of the benchmark configurations (spiral pitch / thickness / intensities).
SPIRAL_CONFIG1 = dict(pitch=12, thickness=3, sheet_mean=170, sheet_sd=15, bg_mean=40, bg_sd=10, blur_sigma=1.0,
                      speckle_sd=0.0)
SPIRAL_CONFIG3 = dict(SPIRAL_CONFIG1, pitch=16, speckle_sd=8.0)
SPIRAL_CONFIG5 = dict(SPIRAL_CONFIG1, pitch=14)


def _sig(lib, name, res, args):
    f = getattr(lib, name)
    f.restype = res
    f.argtypes = args


def lib():
    """Load libfenix_b200.so (building is done by ``fenix_b200.build``); raise if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("FENIX_B200_LIB", LIB_PATH))
    if not path.exists():
        raise FileNotFoundError(f"{path} not built: run `python -m fenix_b200.build` (or __graft_entry__.build())")
    L = C.CDLL(str(path))
    vp, i64, i32, f32p, u8p = C.c_void_p, C.c_int64, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_uint8)
    _sig(L, "fx_last_error", C.c_char_p, [])
    _sig(L, "fx_device_count", i32, [])
    _sig(L, "fx_net_create", i32, [C.c_char_p, i32, i32, i32, i32, C.POINTER(vp)])
    _sig(L, "fx_net_destroy", None, [vp])
    _sig(L, "fx_net_patch", i32, [vp])
    _sig(L, "fx_predict_volume_dev", i32, [vp, vp, i64, i64, i64, C.POINTER(InferOpts), vp, vp, vp])
    _sig(L, "fx_net_create_tiled", i32, [C.c_char_p, C.POINTER(i32), i32, i32, i32, C.POINTER(vp)])
    _sig(L, "fx_net_tile", i32, [vp, C.POINTER(i32), C.POINTER(i32), i32])
    _sig(L, "fx_net_max_batch", i32, [vp])
    _sig(L, "fx_net_classes", i32, [vp])
    _sig(L, "fx_net_features", i32, [vp, C.POINTER(C.c_int), i32])
    _sig(L, "fx_net_calibrate", i32, [vp, u8p, i32])
    _sig(L, "fx_net_set_norm", i32, [vp, i32])
    _sig(L, "fx_net_act_scales", i32, [vp, f32p, i32])
    _sig(L, "fx_net_set_act_scales", i32, [vp, f32p, i32])
    _sig(L, "fx_net_set_layer_precision", i32, [vp, C.POINTER(C.c_int), i32])
    _sig(L, "fx_net_layer_precision", i32, [vp, C.POINTER(C.c_int), C.POINTER(C.c_double), i32])
    _sig(L, "fx_net_layer_name", C.c_char_p, [vp, i32])
    _sig(L, "fx_net_calibrate_schedule", i32, [vp, u8p, i32, C.c_double, C.c_double, C.POINTER(C.c_double),
                                               C.POINTER(C.c_double)])
    _sig(L, "fx_shard_plan", i32, [i64, i64, i64, i32, C.c_double, i32, vp])
    _sig(L, "fx_ipc_buffer_alloc", i32, [i32, C.c_uint64, C.POINTER(vp), vp])
    _sig(L, "fx_ipc_buffer_free", i32, [i32, vp])
    _sig(L, "fx_ipc_open", i32, [i32, vp, C.POINTER(vp)])
    _sig(L, "fx_ipc_close", i32, [i32, vp])
    _sig(L, "fx_predict_volume_multi", i32, [C.POINTER(vp), i32, u8p, i64, i64, i64, C.POINTER(InferOpts), f32p, u8p])
    _sig(L, "fx_net_forward", i32, [vp, vp, i32, vp, i32, i32, vp])
    _sig(L, "fx_predict_volume", i32, [vp, u8p, i64, i64, i64, C.POINTER(InferOpts), f32p, u8p])
    _sig(L, "fx_predict_tiles_dev", i32, [vp, vp, i64, i64, i64, i64, i64, C.POINTER(InferOpts), i64, i64, vp, vp])
    _sig(L, "fx_accum_add", i32, [vp, vp, i64, vp])
    _sig(L, "fx_net_device_status", i32, [vp])
    _sig(L, "fx_selftest_wait_timeout", i32, [i32, C.c_uint64, C.POINTER(C.c_uint32)])
    _sig(L, "fx_tile_starts", i64, [i64, i32, C.c_double, C.POINTER(C.c_int64), i64])
    _sig(L, "fx_gaussian1d", None, [i32, f32p])
    _sig(L, "fx_weight_profile", None, [f32p, i32, C.POINTER(C.c_int64), i64, i64, i64, i64, f32p])
    _sig(L, "fx_norm_tiles", i32, [vp, i64, i64, i64, C.POINTER(C.c_int64), i32, i32, vp, vp])
    _sig(L, "fx_norm_tiles_mode", i32, [vp, i64, i64, i64, C.POINTER(C.c_int64), i32, i32, i32, vp, vp])
    _sig(L, "fx_norm_tiles_noalloc", i32, [vp, i64, i64, i64, C.POINTER(C.c_int64), i32, i32, vp, vp])
    i64p = C.POINTER(C.c_int64)
    _sig(L, "fx_gaccum_create", i32, [i64p, i64p, i32, C.c_double, i64, i32, C.POINTER(vp)])
    _sig(L, "fx_gaccum_destroy", None, [vp])
    for n in ("fx_gaccum_chunk_rows", "fx_gaccum_floor_row", "fx_gaccum_window_planes", "fx_gaccum_tile_rows"):
        _sig(L, n, i64, [vp])
    _sig(L, "fx_gaccum_row_start", i64, [vp, i64])
    _sig(L, "fx_gaccum_set_floor_row", i32, [vp, i64])
    _sig(L, "fx_gaccum_scatter", i32, [vp, i64, i64, i64, f32p])
    _sig(L, "fx_gaccum_predict_row", i32, [vp, vp, i64, u8p, C.POINTER(InferOpts)])
    _sig(L, "fx_gaccum_finalize_below", i32, [vp, i64, u8p, i64, i64p])
    _sig(L, "fx_gaccum_export_planes", i32, [vp, i64, i64, vp])
    _sig(L, "fx_gaccum_add_planes", i32, [vp, i64, i64, vp])
    _sig(L, "fx_gaccum_discard_below", i32, [vp, i64])
    _sig(L, "fx_conv3d", i32, [vp, i32, i32, i32, i32, i32, vp, i32, i32, i32, vp, vp, vp])
    _sig(L, "fx_conv_transpose2", i32, [vp, i32, i32, i32, i32, i32, vp, vp, i32, i32, vp, vp])
    _sig(L, "fx_accum_finalize", i32, [vp, i64, i64, i64, i64, i64, vp, vp, vp, vp, vp, vp])
    _sig(L, "fx_net_profile", i32, [vp, i32])
    _sig(L, "fx_net_profile_read", i32, [vp, C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(C.c_double),
                                         C.POINTER(C.c_int64), C.POINTER(C.c_double), i32])
    _sig(L, "fx_net_profile_read_layers", i32, [vp, C.POINTER(C.c_double), i32])
    _sig(L, "fx_kernel_launches", C.c_ulonglong, [])
    _sig(L, "fx_tc_peak", i32, [i32, i32, C.c_double, i32, C.POINTER(C.c_double), C.POINTER(C.c_double)])
    _sig(L, "fx_tc_rate", i32, [i32, i32, i32, C.c_double, i32, C.POINTER(C.c_double), C.POINTER(C.c_double)])
    _sig(L, "fx_synth_spiral", i32, [u8p, i64, i64, i64, C.POINTER(SpiralParams), C.c_uint64, i64, i64])
    _sig(L, "fx_synth_spiral_chunked", i32, [u8p, i64, i64, i64, C.POINTER(SpiralParams), C.c_uint64, i64, i64])
    _sig(L, "fx_synth_papyrus", i32, [u8p, u8p, i64, i64, i64, C.POINTER(PapyrusParams), C.c_uint64, i64])
    u64p, u32p = C.POINTER(C.c_uint64), C.POINTER(C.c_uint32)
    _sig(L, "fx_fxvol_open", i32, [C.c_char_p, C.POINTER(vp)])
    _sig(L, "fx_fxvol_create", i32, [C.c_char_p, i64, i64, i64, C.c_float, i32, C.POINTER(vp)])
    _sig(L, "fx_fxvol_get_info", i32, [vp, vp])
    _sig(L, "fx_fxvol_chunk_payload", i32, [vp, i32, i64, i64, i64, C.POINTER(C.c_int), C.POINTER(vp), u64p])
    _sig(L, "fx_fxvol_write_chunk_payload", i32, [vp, i32, i64, i64, i64, vp, C.c_uint64])
    _sig(L, "fx_fxvol_set_nlods", i32, [vp, C.c_uint32])
    _sig(L, "fx_fxvol_close", i32, [vp])
    _sig(L, "fx_fxvol_read_volume_u8", i32, [vp, i32, u8p])
    _sig(L, "fx_fxvol_write_volume_u8", i32, [vp, u8p, i32])
    _sig(L, "fx_fxvol_decode_tiles", i32, [vp, C.c_uint64, u64p, u32p, i64, C.c_float, C.c_float, C.c_float, i32,
                                           vp, vp])
    _sig(L, "fx_fxvol_encode_tiles", i32, [vp, vp, i64, C.c_float, C.c_float, C.c_float, i32, vp, C.c_uint64, u64p,
                                           u32p])
    _sig(L, "fx_predict_fxvol", i32, [vp, C.c_char_p, C.c_char_p, C.POINTER(InferOpts), C.c_float])
    _lib = L
    return L


def check(code: int) -> None:
    if code != FX_OK:
        raise FxError(code, lib().fx_last_error().decode())


def _f32(a: np.ndarray):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- tiling math (host) --------------------------------------------------------------------
def tile_starts(dim: int, patch: int, overlap: float) -> np.ndarray:
    L = lib()
    n = L.fx_tile_starts(dim, patch, overlap, None, 0)
    out = np.zeros(n, dtype=np.int64)
    L.fx_tile_starts(dim, patch, overlap, out.ctypes.data_as(C.POINTER(C.c_int64)), n)
    return out


def gaussian1d(n: int) -> np.ndarray:
    out = np.zeros(n, dtype=np.float32)
    lib().fx_gaussian1d(n, out.ctypes.data_as(C.POINTER(C.c_float)))
    return out


def weight_profile(g: np.ndarray, patch: int, starts: np.ndarray, c0: int, cn: int, dim: int) -> np.ndarray:
    g = _f32(g)
    st = np.ascontiguousarray(starts, dtype=np.int64)
    out = np.zeros(cn, dtype=np.float32)
    lib().fx_weight_profile(
        g.ctypes.data_as(C.POINTER(C.c_float)),
        patch,
        st.ctypes.data_as(C.POINTER(C.c_int64)),
        len(st),
        c0,
        cn,
        dim,
        out.ctypes.data_as(C.POINTER(C.c_float)),
    )
    return out


def synth_spiral(shape, seed: int, params: dict | None = None, z_begin: int = 0, z_end: int | None = None,
                 chunked: bool = False, out: np.ndarray | None = None) -> np.ndarray:
    """Spiral-sheet synthetic CT [z_end-z_begin][dy][dx] u8 (deterministic; see fenix_b200_synth.h).
    chunked: noise keyed per 64^3 chunk (fx_synth_spiral_chunked). out: an optional C-contiguous
    u8 destination of that shape (e.g. a view of pinned memory)."""
    dz, dy, dx = shape
    z_end = dz if z_end is None else z_end
    p = SpiralParams(**(params or SPIRAL_CONFIG1))
    if out is None:
        out = np.empty((z_end - z_begin, dy, dx), dtype=np.uint8)
    elif out.shape != (z_end - z_begin, dy, dx) or out.dtype != np.uint8 or not out.flags.c_contiguous:
        raise ValueError("synth_spiral: out must be a C-contiguous u8 array of the output's shape")
    fn = lib().fx_synth_spiral_chunked if chunked else lib().fx_synth_spiral
    rc = fn(out.ctypes.data_as(C.POINTER(C.c_uint8)), dz, dy, dx, C.byref(p), seed, z_begin, z_end)
    if rc != 0:
        raise ValueError("fx_synth_spiral: bad arguments")
    return out


def synth_papyrus(shape, seed: int, stack: int = 0, params: dict | None = None, want_ink: bool = False):
    """Papyrus layer stack [dz][dy][dx] u8 number `stack` of a seeded series (fx_synth_papyrus);
    with want_ink, also its [dy][dx] ink mask."""
    dz, dy, dx = shape
    p = PapyrusParams(**(params or PAPYRUS_INK))
    out = np.empty((dz, dy, dx), dtype=np.uint8)
    ink = np.empty((dy, dx), dtype=np.uint8) if want_ink else None
    rc = lib().fx_synth_papyrus(out.ctypes.data_as(C.POINTER(C.c_uint8)),
                                ink.ctypes.data_as(C.POINTER(C.c_uint8)) if want_ink else None, dz, dy, dx,
                                C.byref(p), seed, stack)
    if rc != 0:
        raise ValueError("fx_synth_papyrus: bad arguments")
    return (out, ink) if want_ink else out


def kernel_launches() -> int:
    """Kernel launches issued by libfenix_b200 in this process."""
    return int(lib().fx_kernel_launches())


def tc_peak(precision: str = "fp8", ms_per_run: float = 50.0, runs: int = 10, device: int = 0):
    """Measured dense tensor rate (TFLOP/s) of this library's MMA-loop kernel: (best, mean) over runs."""
    b, m = C.c_double(), C.c_double()
    check(lib().fx_tc_peak(device, PRECISIONS[precision], ms_per_run, runs, C.byref(b), C.byref(m)))
    return b.value, m.value


def tc_rate(precision: str = "fp8", n_cols: int = 256, ms_per_run: float = 50.0, runs: int = 10, device: int = 0):
    """Measured tensor rate (TFLOP/s) of M = 128 x N = n_cols MMAs: the ceiling of that MMA shape."""
    b, m = C.c_double(), C.c_double()
    check(lib().fx_tc_rate(device, PRECISIONS[precision], n_cols, ms_per_run, runs, C.byref(b), C.byref(m)))
    return b.value, m.value


def device_count() -> int:
    return lib().fx_device_count()


# ---- nets ----------------------------------------------------------------------------------
class Net:
    """A UNet on one GPU (fx_net). ``precision`` is "f16", "bf16" or "fp8". ``patch`` is the side of
    a cubic tile, or a (z, y, x) tile (fx_net_create_tiled); ``self.patch`` is None for a non-cubic
    tile and ``self.tile`` always holds the three extents."""

    def __init__(self, weights_path: str, patch, max_batch: int = 1, precision: str = "bf16", device: int = 0):
        L = lib()
        h = C.c_void_p()
        prec = PRECISIONS[precision]
        tile = (int(patch),) * 3 if np.isscalar(patch) else tuple(int(v) for v in patch)
        if len(tile) != 3:
            raise ValueError("patch: an int or a (z, y, x) triple")
        if tile[0] == tile[1] == tile[2]:
            check(L.fx_net_create(str(weights_path).encode(), tile[0], max_batch, prec, device, C.byref(h)))
        else:
            check(L.fx_net_create_tiled(str(weights_path).encode(), (C.c_int * 3)(*tile), max_batch, prec, device,
                                        C.byref(h)))
        self._h = h
        self.tile = tile
        self.patch = tile[0] if tile[0] == tile[1] == tile[2] else None
        self.precision = precision
        self.device = device

    def stage_masks(self) -> list[int]:
        """Per stage, the axes its strided conv halves (bit 2 z, bit 1 y, bit 0 x; stage 0: 0)."""
        m = (C.c_int * 16)()
        n = lib().fx_net_tile(self._h, None, m, 16)
        return list(m[:n])

    def _opts(self, overlap, channel, sigmoid, batch, tta, norm=0, skip=0, stacks=1):
        opts = InferOpts(self.patch or 0, overlap, channel, sigmoid, batch, tta, norm, skip)
        if self.patch is None:
            opts.tile[:] = list(self.tile)
        opts.stacks = stacks
        return opts

    def predict_volume_dev(self, dev_vol_ptr: int, shape, dev_prob_ptr: int | None, dev_u8_ptr: int | None,
                           overlap: float = 0.5, batch: int = 1, channel: int = 1, sigmoid: int = 0, stacks: int = 1,
                           stream: int | None = None) -> None:
        """fx_predict_volume_dev: device u8 volume in, device f32 map and/or u8 out, asynchronous on
        `stream`. ``stacks`` > 1: the volume is that many independent stacks along z."""
        opts = self._opts(overlap, channel, sigmoid, batch, 0, stacks=stacks)
        self._keep_opts = opts  # the call is asynchronous; the options are read before it returns
        check(lib().fx_predict_volume_dev(self._h, dev_vol_ptr, *shape, C.byref(opts), dev_prob_ptr, dev_u8_ptr, stream))

    def close(self):
        if getattr(self, "_h", None):
            lib().fx_net_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    @property
    def classes(self) -> int:
        return lib().fx_net_classes(self._h)

    @property
    def max_batch(self) -> int:
        return lib().fx_net_max_batch(self._h)

    def features(self) -> list[int]:
        buf = (C.c_int * 16)()
        n = lib().fx_net_features(self._h, buf, 16)
        return list(buf[:n])

    def set_norm(self, norm) -> None:
        """Input normalisation ("zscore", "pct_minmax", "unit255" or its fx_norm code) that
        calibrate, calibrate_schedule and forward apply to u8 tiles (default zscore)."""
        check(lib().fx_net_set_norm(self._h, NORMS[norm] if isinstance(norm, str) else int(norm)))

    def calibrate(self, patches_u8: np.ndarray) -> None:
        p = np.ascontiguousarray(patches_u8, dtype=np.uint8)
        check(lib().fx_net_calibrate(self._h, p.ctypes.data_as(C.POINTER(C.c_uint8)), p.shape[0]))

    def set_act_scales(self, scales) -> None:
        s = np.ascontiguousarray(scales, dtype=np.float32)
        check(lib().fx_net_set_act_scales(self._h, s.ctypes.data_as(C.POINTER(C.c_float)), len(s)))

    def act_scales(self) -> np.ndarray:
        buf = np.zeros(256, dtype=np.float32)
        n = lib().fx_net_act_scales(self._h, buf.ctypes.data_as(C.POINTER(C.c_float)), 256)
        return buf[:n]

    def layers(self) -> list[dict]:
        """Conv layers in act_scales order: weights prefix, operand precision it runs with and
        algorithmic FLOPs per tile."""
        cap = 256
        q = (C.c_int * cap)()
        f = (C.c_double * cap)()
        n = lib().fx_net_layer_precision(self._h, q, f, cap)
        names = {0: "bf16", 1: "fp8", 2: "f16"}
        return [{"name": lib().fx_net_layer_name(self._h, i).decode(), "precision": names[q[i]], "flops": f[i]}
                for i in range(n)]

    def calibrate_schedule(self, patches_u8: np.ndarray, min_dice: float = 0.99, max_abs: float = 0.0):
        """fp8 nets: choose which layers run e4m3 from calibration patches (fx_net_calibrate_schedule);
        returns (Dice, max |dp|) of the schedule against the net's 16-bit forward."""
        p = np.ascontiguousarray(patches_u8, dtype=np.uint8)
        d, m = C.c_double(), C.c_double()
        check(lib().fx_net_calibrate_schedule(self._h, p.ctypes.data_as(C.POINTER(C.c_uint8)), p.shape[0], min_dice,
                                              max_abs, C.byref(d), C.byref(m)))
        return d.value, m.value

    def set_layer_precision(self, precisions) -> None:
        """fp8 nets: per conv layer (act_scales order) "fp8" or the 16-bit type ("f16")."""
        v = (C.c_int * len(precisions))(*[PRECISIONS[p] for p in precisions])
        check(lib().fx_net_set_layer_precision(self._h, v, len(precisions)))

    def profile(self, enable: bool) -> None:
        check(lib().fx_net_profile(self._h, 1 if enable else 0))

    def profile_read(self, per_launch_cap: int = 4096) -> dict:
        ms, fl, f8 = C.c_double(), C.c_double(), C.c_double()
        n = C.c_int64()
        per = np.zeros(2 * per_launch_cap, dtype=np.float64)
        check(lib().fx_net_profile_read(self._h, C.byref(ms), C.byref(fl), C.byref(f8), C.byref(n),
                                        per.ctypes.data_as(C.POINTER(C.c_double)), per_launch_cap))
        k = min(n.value, per_launch_cap)
        return {"conv_ms": ms.value, "conv_flops": fl.value, "fp8_flops": f8.value, "conv_launches": n.value,
                "per_launch": per[: 2 * k].reshape(k, 2)}

    def profile_read_layers(self) -> list[dict]:
        """The profiled conv time per layer (fx_net_profile_read_layers), with each layer's name,
        precision and algorithmic FLOPs per tile; clears the record."""
        buf = np.zeros(1024, dtype=np.float64)
        n = lib().fx_net_profile_read_layers(self._h, buf.ctypes.data_as(C.POINTER(C.c_double)), 1024)
        if n < 0:
            raise FxError(8, lib().fx_last_error().decode())
        return [dict(l, ms=float(buf[i])) for i, l in enumerate(self.layers()[:n])]

    def forward_dev(self, dev_tiles_ptr: int, nb: int, dev_prob_ptr: int, channel: int = 1, sigmoid: int = 0,
                    stream: int | None = None) -> None:
        check(lib().fx_net_forward(self._h, dev_tiles_ptr, nb, dev_prob_ptr, channel, sigmoid, stream))

    def predict_volume(self, vol_u8: np.ndarray, overlap: float = 0.5, batch: int = 1, channel: int = 1,
                       sigmoid: int = 0, want_prob: bool = True, want_u8: bool = True, tta: int = 0,
                       norm: str = "zscore", skip_constant: bool = False, core=None, tile_filter=None,
                       stacks: int = 1, ckpt_path=None, ckpt_every: int = 128, weights_hash: int = 0,
                       input_hash: int = 0):
        """core = (z, y, x, dz, dy, dx) output crop (extents <= 0: to the end); tile_filter =
        callable(z0, y0, x0, patch) -> bool. Outputs have the crop's dims when cropped."""
        v = np.ascontiguousarray(vol_u8, dtype=np.uint8)
        dz, dy, dx = v.shape
        opts = self._opts(overlap, channel, sigmoid, batch, tta, NORMS[norm], 1 if skip_constant else 0, stacks)
        if ckpt_path is not None:
            opts.ckpt_path = str(ckpt_path).encode()
            opts.ckpt_every, opts.weights_hash, opts.input_hash = ckpt_every, weights_hash, input_hash
        out_shape = v.shape
        if core is not None:
            opts.core_org[:] = list(core[:3])
            opts.core_ext[:] = list(core[3:])
            out_shape = tuple(min(e, n - o) if e > 0 else n - o
                              for o, e, n in zip((min(max(c, 0), n) for c, n in zip(core[:3], v.shape)), core[3:], v.shape))
        if tile_filter is not None:
            cb = TileFilter(lambda z0, y0, x0, p, _u: 1 if tile_filter(z0, y0, x0, p) else 0)
            opts.tile_filter = cb
        prob = np.zeros(out_shape, dtype=np.float32) if want_prob else None
        u8 = np.zeros(out_shape, dtype=np.uint8) if want_u8 else None
        check(
            lib().fx_predict_volume(
                self._h,
                v.ctypes.data_as(C.POINTER(C.c_uint8)),
                dz,
                dy,
                dx,
                C.byref(opts),
                prob.ctypes.data_as(C.POINTER(C.c_float)) if prob is not None else None,
                u8.ctypes.data_as(C.POINTER(C.c_uint8)) if u8 is not None else None,
            )
        )
        return prob, u8

    def predict_fxvol(self, in_path, out_path, overlap: float = 0.5, batch: int = 1, channel: int = 1,
                      sigmoid: int = 0, tta: int = 0, out_q: float = 32.0) -> None:
        """predict-surface over archives: u8 .fxvol in, u8 .fxvol (q = out_q, LOD pyramid) out."""
        opts = InferOpts(self.patch, overlap, channel, sigmoid, batch, tta)
        check(lib().fx_predict_fxvol(self._h, str(in_path).encode(), str(out_path).encode(), C.byref(opts), out_q))

    def predict_tiles_dev(self, dev_slab_ptr: int, slab_shape, z_origin: int, full_dz: int, overlap: float,
                          batch: int, tile_begin: int, tile_end: int, dev_acc_ptr: int, channel: int = 1,
                          sigmoid: int = 0, stream: int | None = None, tta: int = 0) -> None:
        dz, dy, dx = slab_shape
        opts = InferOpts(self.patch, overlap, channel, sigmoid, batch, tta)
        check(lib().fx_predict_tiles_dev(self._h, dev_slab_ptr, dz, dy, dx, z_origin, full_dz, C.byref(opts),
                                         tile_begin, tile_end, dev_acc_ptr, stream))


def default_stream_ptr():
    """The current torch CUDA stream as a raw pointer (torch is only plumbing here)."""
    import torch

    return torch.cuda.current_stream().cuda_stream
