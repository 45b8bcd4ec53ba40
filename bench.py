#!/usr/bin/env python3
"""Benchmark: fp8 3D-UNet sliding-window inference over a 1024^3 u8 volume on 1..8 B200.

Workload (the benchmark configuration): the 5-stage plain UNet (32/64/128/256/320, 2 convs +
InstanceNorm + LeakyReLU per stage, stride-2 conv down, ConvTranspose 2^3 up, 1x1x1 head to 2
classes + softmax), random Kaiming init (seed 1), fp8 e4m3 operands with per-output-channel weight
scales and per-tensor activation scales calibrated on 4 seeded patches; a synthetic 1024^3 u8
spiral-sheet volume (pitch 16, thickness 3, N(0,8) speckle, seed 2); 128^3 tiles at overlap 0.5
(3375 tiles) with Gaussian blending, normalised and encoded to u8. One step = one full pass over
the volume. Multi-GPU: the volume is split into z-slabs by tile ranges (fenix_b200/shard.py); each
owner reads the tile-overlap bands its neighbours accumulated straight from their HBM over NVLink
(CUDA IPC mappings, an add kernel doing the loads) and finalises the planes it owns. The ranks'
process group is gloo (host barriers and the timing reduction); nothing goes through NCCL.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl fenix|reference] [--precision fp8|fp8-all|f16|bf16]

--precision fp8 (the default) is the calibrated mixed schedule: e4m3 operands in the layers the
calibration picks (fx_net_calibrate_schedule, Dice >= 0.993 against the net's 16-bit forward on the
4 calibration patches), f16 in the rest; fp8-all puts every layer that can take e4m3 on it.

For N > 1 launch one process per GPU with torch.distributed.run. Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Mvoxels/s fp8 3D-UNet sliding-window inference @1/2/4/8 B200; % tcgen05 peak"
FEATURES = (32, 64, 128, 256, 320)
INK_FEATURES_B = (64, 128, 256, 512)  # the layer-stack net (fenix_b200.weights.INK_*), restated for the
INK_STRIDES_B = ((1, 1, 1), (1, 2, 2), (1, 2, 2), (2, 2, 2))  # reference arm, which imports no product code
WEIGHT_SEED, VOLUME_SEED, CALIB_SEED0 = 1, 2, 1000
SCHED_DICE = 0.993  # the fp8 schedule's agreement with the 16-bit forward on the calibration patches
PARITY_CASE = ROOT / "tests" / "golden" / "net128_cfg3.npz"  # the reference's map of a 192^3 crop
# DRAM traffic of the 22 conv launches of one fp8 forward, per 128^3 tile (dram__bytes_read.sum +
# dram__bytes_write.sum from an ncu launch list of `bench.py --size 256 --steps 1 --warmup 3`:
# 4.563 GB read + 5.933 GB written per forward of 8 tiles). ncu cannot run inside the timed bench,
# so the captured figure is carried here and re-captured when the conv kernel changes.
CONV_DRAM_BYTES_PER_TILE = 1.2946e9  # ncu launch list of the 256^3 bench: (112.121 + 137.737) GB over 193 tiles
# The same for the calibrated schedule (--precision fp8, the default): the 22 conv launches of the
# first forward of `bench.py --size 256 --steps 1 --warmup 3 --minimal --batch 4` (4 tiles),
# 3.935 GB read + 2.722 GB written.
CONV_DRAM_BYTES_PER_TILE_SCHED = 1.6644e9


def env_int(name, default):
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


def peaks():
    """Roofline denominators: MEASURED_PEAKS.json (driver-written) or the recipe's fallback."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), float(d["hbm_gbs"]), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region (200 ms period)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.rows = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if "Active" in r[5 + i] and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def ref_crop(S, ext, seed=VOLUME_SEED):
    """The central ext^3 crop of the S^3 benchmark volume, made on the checker side (oracle/synth.c,
    byte-identical to the product's generator) so a reference process never loads the product."""
    from oracle import oracle as orc

    o = (S - ext) // 2
    slab = orc.synth_spiral((S, S, S), seed, orc.SPIRAL_CONFIG3, o, o + ext)
    return np.ascontiguousarray(slab[:, o:o + ext, o:o + ext]), o


def cpu_reference(weights, vol, P, overlap, threads=None):
    """The reference's own CPU inference (oracle/_ref/ref_infer: predict_surface_filled + ConvStack via
    libtorch, fp32, all host threads) over `vol`. Returns (seconds per tile, threads, tiles, seconds)."""
    from oracle import oracle as orc

    _, info = orc.ref_infer(weights, vol, P, overlap, batch=2, threads=threads or os.cpu_count())
    return info["seconds"] / info["tiles"], int(info["threads"]), int(info["tiles"]), float(info["seconds"])


def workload_config(args, tiles, world):
    S, P = args.size, args.patch
    return {
        "workload": f"fp8 sliding-window inference, {S}^3 u8 volume, {P}^3 tiles, overlap {args.overlap}, "
                    f"{tiles} tiles, Gaussian blend, u8 output; 5-stage UNet 32/64/128/256/320",
        "volume": [S, S, S], "patch": P, "overlap": args.overlap, "tiles": tiles, "batch": args.batch,
        "precision": args.precision, "parallelism": f"z-slab x{world}",
        "l2": f"inputs larger than L2: {S}^3 u8 volume + {S}^3 f32 accumulator per step",
    }


def run_reference_arm(args):
    """The reference's own CPU implementation of the path (oracle/_ref/ref_infer, compiled from the
    reference's sources), all host threads, on this workload. Imports only the checker side
    (oracle/): the volume, the network file and the tile grid are made without the product library.
    Each warm-up step runs one 128^3 tile; each timed step runs the next tile of the 27-tile grid of
    the volume's central 256^3 crop (cycling), and the rate is the per-tile time projected over the
    full volume's tile grid (the reference runs its tiles one after another)."""
    rank = env_int("RANK", 0)
    if rank != 0:
        return 0
    from oracle import netgen
    from oracle import oracle as orc

    ex = ROOT / "oracle" / "_ref" / "ref_infer"
    if not ex.exists():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/ref_infer not built (needs the reference tree at build time)"}))
        return 0
    S, P = args.size, args.patch
    tiles = len(orc.tile_starts(S, P, args.overlap)) ** 3
    ext = min(S, 2 * P)
    crop, o = ref_crop(S, ext)
    st = orc.tile_starts(ext, P, args.overlap)
    origins = [(z, y, x) for z in st for y in st for x in st]
    thr = os.cpu_count() or 1
    with tempfile.TemporaryDirectory() as td:
        w = netgen.make_plain_unet(Path(td) / "w.fxweights", FEATURES, seed=WEIGHT_SEED)
        t0 = crop[:P, :P, :P]
        for _ in range(args.warmup):
            cpu_reference(w, t0, P, args.overlap, thr)
        times = []
        for k in range(args.steps):
            z, y, x = origins[k % len(origins)]
            per_tile, used, _, _ = cpu_reference(w, np.ascontiguousarray(crop[z:z + P, y:y + P, x:x + P]), P,
                                                 args.overlap, thr)
            times.append(per_tile)
    per_tile = sum(times) / len(times)
    value = S ** 3 / (tiles * per_tile) / 1e6
    sample = (f"reference predict_surface_filled (libtorch fp32, {used} threads), one {P}^3 tile per step: the "
              f"tiles of the {len(origins)}-tile grid of the central {ext}^3 crop [{o}, {o + ext})^3 of the {S}^3 "
              f"volume in turn ({args.steps} steps, mean {per_tile:.3f} s per tile); rate projected over the "
              f"volume's {tiles} tiles")
    line = {"metric": METRIC, "value": value, "unit": "Mvoxels/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_tile * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, tiles, args.gpus),
            "cpu_baseline": {"value": value, "unit": "Mvoxels/s", "cores": used, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": value, "unit": "Mvoxels/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def fxvol_measure(vol_u8: np.ndarray, pred_u8: np.ndarray, tmp: str, reps: int = 2) -> dict:
    """The .fxvol IO either side of the path, timed end to end through the C ABI (host volume <->
    archive file, chunks decoded / encoded on the GPU): the input volume read from an archive at the
    reference's default q = 8 (predict-surface's .fxvol input, inference.cpp:553-567) and the u8
    prediction written at q = 32 with its LOD pyramid (inference.cpp:343-356). The reference's own
    VolumeArchive (oracle/_ref/ref_fxvol, all host threads) is timed on the same files."""
    import fenix_b200.fxvol as fv

    inp, out = Path(tmp) / "in.fxvol", Path(tmp) / "pred.fxvol"
    with fv.VolumeArchive.create(inp, vol_u8.shape, 8.0) as a:
        a.write_volume_u8(vol_u8)

    def best(fn):
        ts = []
        for _ in range(reps + 1):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return min(ts[1:])

    def write():
        with fv.VolumeArchive.create(out, pred_u8.shape, 32.0) as a:
            a.write_volume_u8(pred_u8)

    def read():
        with fv.VolumeArchive.open(inp) as a:
            a.read_volume_u8()

    t_w, t_r = best(write), best(read)
    vox = float(vol_u8.size)
    res = {
        "unit": "Gvoxels/s",
        "decode": {"value": vox / t_r / 1e9, "s": t_r, "archive_bytes": inp.stat().st_size, "q": 8.0,
                   "what": "fx_fxvol_read_volume_u8: LOD-0 read of the input volume's archive"},
        "encode": {"value": vox / t_w / 1e9, "s": t_w, "archive_bytes": out.stat().st_size, "q": 32.0,
                   "what": "fx_fxvol_write_volume_u8: the u8 prediction, LOD 0 + pyramid"},
    }
    tool = ROOT / "oracle" / "_ref" / "ref_fxvol"
    if tool.exists():
        raw = Path(tmp) / "pred.raw"
        pred_u8.tofile(raw)
        thr = os.cpu_count() or 1
        env = dict(os.environ, OMP_NUM_THREADS=str(thr))
        dz, dy, dx = pred_u8.shape
        t0 = time.perf_counter()
        subprocess.run([str(tool), "read", str(inp), str(Path(tmp) / "back.raw")], check=True, env=env,
                       capture_output=True)
        t_cr = time.perf_counter() - t0
        t0 = time.perf_counter()
        subprocess.run([str(tool), "write", "32", str(dz), str(dy), str(dx), str(raw), str(Path(tmp) / "cpu.fxvol")],
                       check=True, env=env, capture_output=True)
        t_cw = time.perf_counter() - t0
        res["cpu_baseline"] = {"kind": "reference", "cores": thr, "decode": vox / t_cr / 1e9,
                               "encode": vox / t_cw / 1e9, "unit": "Gvoxels/s",
                               "sample": "the same two archives, one run each, process wall time"}
    return res


def measure_tc_peaks(fx, device):
    """Dense tcgen05 rates of this GPU from fx_tc_peak, with the SM clock seen during the sustained runs."""
    out = {}
    for kind, prec in (("e4m3", "fp8"), ("f16", "f16")):
        burst, _ = fx.tc_peak(prec, 50.0, 10, device)
        clk = ClockSampler(device)
        clk.start()
        sus, _ = fx.tc_peak(prec, 4000.0, 1, device)
        c = clk.stop()
        out[kind] = {"burst": burst, "sustained": sus, "unit": "TFLOP/s", "sustained_sm_mhz": c.get("sm_mhz"),
                     "sustained_reasons": c.get("reasons")}
    return out


def layer_times(net, step, tiles):
    """One more profiled step, summed per conv layer: ms per step, operand type and achieved
    TFLOP/s (algorithmic FLOPs per tile x tiles of the step / the layer's summed launch time)."""
    import torch

    net.profile(True)
    step()
    torch.cuda.synchronize()
    net.profile(False)
    out = []
    for l in net.profile_read_layers():
        out.append({"layer": l["name"], "precision": l["precision"], "ms": round(l["ms"], 3),
                    "tflops": round(l["flops"] * tiles / max(l["ms"], 1e-9) / 1e9, 1)})
    return out


def vox_of(S):
    return float(S) ** 3


def precision_report(net, sched):
    """Which conv layers ran e4m3 and the share of the algorithmic FLOPs they carry."""
    layers = net.layers()
    tot = sum(l["flops"] for l in layers)
    f8 = [l for l in layers if l["precision"] == "fp8"]
    out = {"fp8_layers": [l["name"] for l in f8], "fp8_flop_share": sum(l["flops"] for l in f8) / tot,
           "layers": len(layers)}
    if sched:
        out.update(sched)
    return out


def parity_check(fx, net, batch, precision):
    """The benchmark's net, calibration and schedule on the central 192^3 crop of the same volume,
    against the reference's own CPU inference of that crop (tests/golden/net128_cfg3.npz, every
    voxel): max |dp| and Dice of the 0.5-thresholded masks, beside the bounds the path is held to."""
    g = np.load(PARITY_CASE)
    full, org, shape = (tuple(int(v) for v in g[k]) for k in ("full_shape", "crop_origin", "shape"))
    slab = fx.synth_spiral(full, int(g["volume_seed"]), fx.SPIRAL_CONFIG3, org[0], org[0] + shape[0])
    vol = np.ascontiguousarray(slab[:, org[1]:org[1] + shape[1], org[2]:org[2] + shape[2]])
    prob, _ = net.predict_volume(vol, overlap=float(g["overlap"]), batch=batch, want_u8=False)
    ref = g["prob_u16"].astype(np.float32) / np.float32(65535.0)
    e = np.abs(prob - ref)
    a, b = prob >= 0.5, ref >= 0.5
    dice = float(2.0 * (a & b).sum() / max(int(a.sum() + b.sum()), 1))
    bound = 3e-2 if precision == "fp8" else 1e-2
    return {"case": f"central {shape[0]}^3 crop of the benchmark volume ({len(fx.tile_starts(shape[0], 128, 0.5)) ** 3} "
                    "tiles), reference = its own CPU inference (libtorch fp32), every voxel",
            "max_abs": float(e.max()), "mean_abs": float(e.mean()), "dice": dice,
            "bound_max_abs": bound, "bound_dice": 0.99 if precision == "fp8" else None,
            "meets_max_abs": bool(e.max() <= bound), "meets_dice": bool(dice >= 0.99)}


INK_METRIC = "Mvoxels/s fp8 wide-ink 3D-UNet layer-stack inference @1/2/4/8 B200; % tcgen05 peak"
INK_SHAPE, INK_TILE, INK_OVERLAP, INK_STACKS = (64, 512, 512), (64, 256, 256), 0.25, 8
INK_WEIGHT_SEED, INK_VOLUME_SEED = 3, 3
INK_PARITY_CASE = ROOT / "tests" / "golden" / "ink_small.npz"


def ink_config(world, precision):
    return {
        "workload": f"wide-ink layer stacks: {INK_STACKS} stacks of {'x'.join(map(str, INK_SHAPE))} u8 per GPU, "
                    f"{'x'.join(map(str, INK_TILE))} tiles at overlap {INK_OVERLAP} (1x3x3 per stack), Gaussian blend, "
                    "u8 output; 4-stage UNet 64/128/256/512, stride (1,2,2) at stages 1-2 and 2 at stage 3, "
                    "1 class + sigmoid",
        "stack": list(INK_SHAPE), "tile": list(INK_TILE), "overlap": INK_OVERLAP, "stacks_per_gpu": INK_STACKS,
        "batch": 8, "precision": precision, "parallelism": f"independent stacks x{world}",
        "l2": "inputs larger than L2: 134 MB u8 stacks + 537 MB f32 accumulator per GPU per step",
    }


def ink_cpu_sample(w, threads=None):
    """The C oracle's forward (fp32, OpenMP over all host threads) of one 16 x 64 x 64 tile of the
    same net, projected per voxel to the workload's tiles (the net's FLOPs per tile voxel are within
    1% between the two tile sizes). Returns (seconds per workload tile, threads, seconds)."""
    from oracle import oracle as orc

    n = orc.Net(w)
    x = np.random.default_rng(0).normal(size=(1, 16, 64, 64)).astype(np.float32)
    t0 = time.perf_counter()
    n.forward_tiled(x, channel=0, sigmoid=1)
    secs = time.perf_counter() - t0
    scale = (INK_TILE[0] * INK_TILE[1] * INK_TILE[2]) / (16 * 64 * 64)
    return secs * scale, os.cpu_count() or 1, secs


def run_ink_reference(args):
    """Reference arm of the layer-stack workload. The reference's nets take one int stride per stage
    and its window tiles cubes, so it cannot run this net; the CPU baseline is the C oracle's
    restatement (kind "port"), timed on a bounded sample (one 16 x 64 x 64 tile per step)."""
    if env_int("RANK", 0) != 0:
        return 0
    from oracle import netgen

    with tempfile.TemporaryDirectory() as td:
        w = netgen.make_plain_unet(Path(td) / "w.fxweights", INK_FEATURES_B, ncls=1, seed=INK_WEIGHT_SEED,
                                   strides=INK_STRIDES_B)
        for _ in range(1):
            ink_cpu_sample(w)
        ts = [ink_cpu_sample(w)[0] for _ in range(args.steps)]
    per_tile = sum(ts) / len(ts)
    tiles = INK_STACKS * 9
    value = INK_STACKS * float(np.prod(INK_SHAPE)) / (tiles * per_tile) / 1e6
    thr = os.cpu_count() or 1
    sample = (f"C oracle forward (fp32, {thr} threads) of one 16x64x64 tile per step, projected per voxel to the "
              f"{tiles} 64x256x256 tiles of {INK_STACKS} stacks ({args.steps} steps)")
    print(json.dumps({"metric": INK_METRIC, "value": value, "unit": "Mvoxels/s", "impl": "reference",
                      "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": per_tile * tiles * 1e3, "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": ink_config(args.gpus, "f32"),
                      "cpu_baseline": {"value": value, "unit": "Mvoxels/s", "cores": thr, "kind": "port",
                                       "sample": sample},
                      "e2e": {"value": value, "unit": "Mvoxels/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
    return 0


def ink_parity(fx, wdir, precision, sched_dice):
    """The workload's net (same weights) on the small layer stack of tests/golden/ink_small.npz in
    16 x 64 x 64 tiles, against the C oracle's full map: max |dp| and Dice, 16-bit and the
    calibrated schedule picked the same way as for the benchmark net."""
    from fenix_b200.weights import make_plain_unet

    g = np.load(INK_PARITY_CASE)
    tile = tuple(int(v) for v in g["tile"])
    w = make_plain_unet(Path(wdir) / "ink_small.fxweights", INK_FEATURES_B, ncls=1, seed=int(g["weight_seed"]),
                        strides=INK_STRIDES_B)
    vol = fx.synth_papyrus(tuple(int(v) for v in g["shape"]), int(g["volume_seed"]), int(g["stack"]))
    ref = g["prob_u16"].astype(np.float32) / np.float32(65535.0)
    out = {"case": f"{'x'.join(str(int(v)) for v in g['shape'])} papyrus stack in {'x'.join(map(str, tile))} tiles, "
                   "reference = the C oracle's fp32 sliding window (the reference has no anisotropic net), every voxel"}
    for tag, prec in (("f16", "f16"), ("schedule", "fp8")):
        if tag == "schedule" and precision != "fp8":
            continue
        net = fx.Net(w, tile, max_batch=8, precision=prec)
        if prec == "fp8":
            cal = np.stack([fx.synth_papyrus(tile, 1000 + i, 0) for i in range(4)])
            net.calibrate_schedule(cal, min_dice=sched_dice)
        prob, _ = net.predict_volume(vol, overlap=float(g["overlap"]), batch=8, channel=0, sigmoid=1, want_u8=False)
        net.close()
        e = np.abs(prob - ref)
        a, b = prob >= 0.5, ref >= 0.5
        out[tag] = {"max_abs": float(e.max()), "mean_abs": float(e.mean()),
                    "dice": float(2.0 * (a & b).sum() / max(int(a.sum() + b.sum()), 1))}
    return out


def run_ink(args):
    """The layer-stack (wide-ink) workload: each GPU predicts a batch of 8 papyrus stacks of
    64 x 512 x 512 in one call (fx_infer_opts.stacks = 8: 72 tiles of 64 x 256 x 256, 9 forwards of
    8), stacks sharded across ranks with no data exchange (weak scaling). value = device-resident
    fx_predict_volume_dev; e2e = fx_predict_volume with pinned host input and u8 output."""
    import ctypes as C

    import torch

    import fenix_b200 as fx
    from fenix_b200.weights import make_plain_unet

    rank, world, local = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    tmp = tempfile.mkdtemp(prefix=f"fxink{rank}_")
    wpath = make_plain_unet(Path(tmp) / "ink.fxweights", INK_FEATURES_B, ncls=1, seed=INK_WEIGHT_SEED,
                            strides=INK_STRIDES_B)
    fp8 = args.precision.startswith("fp8")
    net = fx.Net(wpath, INK_TILE, max_batch=8, precision="fp8" if fp8 else args.precision, device=local)
    sched = None
    if fp8:
        got = [None]
        if rank == 0:
            calib = np.stack([fx.synth_papyrus(INK_TILE, CALIB_SEED0 + i, 0) for i in range(4)])
            net.calibrate(calib)
            if args.precision == "fp8":
                d_cal, m_cal = net.calibrate_schedule(calib, min_dice=SCHED_DICE)
                sched = {"calibration_dice": d_cal, "calibration_max_abs": m_cal, "target_dice": SCHED_DICE}
            got = [(net.act_scales().tolist(), [l["precision"] for l in net.layers()], sched)]
        if world > 1:
            torch.distributed.broadcast_object_list(got, src=0)
            if rank != 0:
                scales, precs, sched = got[0]
                net.set_act_scales(scales)
                net.set_layer_precision(["fp8" if p == "fp8" else "f16" for p in precs])
    dz = INK_SHAPE[0] * INK_STACKS
    shape = (dz,) + INK_SHAPE[1:]
    host = torch.from_numpy(np.concatenate([fx.synth_papyrus(INK_SHAPE, INK_VOLUME_SEED, rank * INK_STACKS + k)
                                            for k in range(INK_STACKS)])).pin_memory()
    host_out = torch.empty(shape, dtype=torch.uint8).pin_memory()
    dv = host.cuda()
    du = torch.empty(shape, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream(device=local)

    def timed(fn, k):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("fx_timed")  # lets a profiler select the timed launches (--nvtx-include)
        ev0.record(stream)
        for _ in range(k):
            fn()
        ev1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        barrier()
        ms = ev0.elapsed_time(ev1)
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def dev_step():
        net.predict_volume_dev(dv.data_ptr(), shape, None, du.data_ptr(), overlap=INK_OVERLAP, batch=8, channel=0,
                               sigmoid=1, stacks=INK_STACKS, stream=stream.cuda_stream)

    opts = net._opts(INK_OVERLAP, 0, 1, 8, 0, stacks=INK_STACKS)
    hv, hu = host.numpy(), host_out.numpy()

    def e2e_step():
        # fx_predict_volume runs on the net's own stream and returns after its D2H copy
        fx.check(fx.lib().fx_predict_volume(net.handle, hv.ctypes.data_as(C.POINTER(C.c_uint8)), *shape,
                                            C.byref(opts), None, hu.ctypes.data_as(C.POINTER(C.c_uint8))))

    for _ in range(args.warmup):
        dev_step()
    torch.cuda.synchronize()
    fx.check(fx.lib().fx_net_device_status(net.handle))
    clocks = ClockSampler(local)
    clocks.start()
    l0 = fx.kernel_launches()
    ms = timed(dev_step, args.steps)
    launches = fx.kernel_launches() - l0
    clk = clocks.stop()
    fx.check(fx.lib().fx_net_device_status(net.handle))
    e2e_step()
    t0 = time.perf_counter()
    barrier()
    for _ in range(args.steps):
        e2e_step()
    barrier()
    ms_e2e = (time.perf_counter() - t0) * 1e3
    if world > 1:
        t = torch.tensor([ms_e2e, float(launches)], dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms_e2e = float(t[0].item())
        launches *= world
    net.profile(True)
    dev_step()
    torch.cuda.synchronize()
    net.profile(False)
    prof = net.profile_read()
    layer_table = layer_times(net, dev_step, float(INK_STACKS * 9))
    vox = float(np.prod(shape)) * world
    value = vox * args.steps / (ms / 1e3) / 1e6
    e2e = vox * args.steps / (ms_e2e / 1e3) / 1e6
    conv_tflops = prof["conv_flops"] / (prof["conv_ms"] / 1e3) / 1e12
    f8 = prof["fp8_flops"] / max(prof["conv_flops"], 1.0)
    cpu = parity = tc = None
    if rank == 0:
        tc = measure_tc_peaks(fx, local)
        if world == 1:
            parity = ink_parity(fx, tmp, "fp8" if fp8 else args.precision, SCHED_DICE) if INK_PARITY_CASE.exists() else None
            if not args.no_cpu_baseline:
                try:
                    per_tile, thr, secs = ink_cpu_sample(wpath)
                    cpu = {"value": INK_STACKS * float(np.prod(INK_SHAPE)) / (INK_STACKS * 9 * per_tile) / 1e6,
                           "unit": "Mvoxels/s", "cores": thr, "kind": "port",
                           "sample": f"C oracle forward (fp32) of one 16x64x64 tile ({secs:.2f} s), projected per voxel "
                                     f"to the {INK_STACKS * 9} 64x256x256 tiles of a step"}
                except Exception as e:
                    cpu = {"value": None, "unit": "Mvoxels/s", "cores": None, "kind": "port", "sample": f"failed: {e}"}

        def mixed(p8, p16):
            return 1.0 / (f8 / p8 + (1.0 - f8) / p16)

        peak = mixed(tc["e4m3"]["sustained"], tc["f16"]["sustained"])
        line = {
            "metric": INK_METRIC, "value": value, "unit": "Mvoxels/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": {"fp8": "e4m3 + f16 (calibrated schedule)", "fp8-all": "e4m3", "f16": "f16", "bf16": "bf16"}[args.precision],
            "data": "synthetic: papyrus layer stacks (fibre texture sigma 4/1/1, 110 +- 20, 5% ink columns +25, seed 3, "
                    "stack k of rank r = series index 8r + k); random-init Kaiming weights (seed 3)",
            "config": ink_config(world, args.precision),
            "roofline": {"bound": "tensor", "achieved": conv_tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": conv_tflops / peak, "traffic": None,
                         "kernel": "conv_tc_kernel (every conv launch of one step, summed)",
                         "peak_source": "fx_tc_peak sustained e4m3 / f16 rates weighted by the step's e4m3 FLOP share",
                         "tc_peaks_measured": tc, "conv_ms_per_step": prof["conv_ms"],
                         "conv_flops_per_step": prof["conv_flops"], "fp8_flop_share": f8,
                         "conv_share_of_step": prof["conv_ms"] / (ms / args.steps),
                         "frac_step": prof["conv_flops"] / (ms / args.steps / 1e3) / 1e12 / peak},
            "precision_schedule": precision_report(net, sched),
            "conv_layers": layer_table,
            "parity": parity,
            "e2e": {"value": e2e, "unit": "Mvoxels/s", "h2d_bytes_per_step": int(np.prod(shape)) * world,
                    "d2h_bytes_per_step": int(np.prod(shape)) * world,
                    "path": "fx_predict_volume (C ABI), pinned host u8 stacks in, u8 out, host-timed per step"},
            "cpu_baseline": cpu, "clocks": clk, "gpu_launches": launches,
        }
        print(json.dumps(line))
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    net.close()
    return 0


STREAM_METRIC = "Mvoxels/s fp8 out-of-core streaming surface inference (finalised u8 output) @1/2/4/8 B200"
STREAM_SHAPE, STREAM_PATCH, STREAM_OVERLAP, STREAM_SEED = (2048, 4096, 4096), 192, 0.5, 4


def run_stream(args):
    """The out-of-core workload: the 2048 x 4096 x 4096 spiral volume with noise keyed per 64^3
    chunk (seed 4, pitch 14), 192^3 tiles at overlap 0.5 (a 21 x 42 x 42 tile grid, 1764 tiles per
    tile row), the benchmark's 5-stage net with the calibrated fp8 schedule, streamed by tile row
    (fenix_b200/stream.py): each GPU takes a contiguous range of the tile rows, copies each row's
    192 input planes from pinned host memory into its device accumulator window, finalises u8
    chunk rows into pinned host memory as soon as no later row reaches them, and the chunk rows a
    range shares with the range below are handed to that rank's GPU over NVLink (CUDA IPC) and
    finalised there. --stream-rows R runs the first R tile rows (default: all 21, the whole
    volume). value = finalised output voxels of all GPUs / the slowest rank's wall time of its
    whole share (host copies included: the workload is the stream). Warm-up: W forwards of 8
    tiles on each GPU."""
    import ctypes as C

    import torch

    import fenix_b200 as fx
    from fenix_b200.stream import StreamRank
    from fenix_b200.weights import make_plain_unet

    rank, world, local = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=1200))
        group = dist.group.WORLD
    P, ov = STREAM_PATCH, STREAM_OVERLAP
    dz, dy, dx = STREAM_SHAPE
    tmp = tempfile.mkdtemp(prefix=f"fxstream{rank}_")
    wpath = make_plain_unet(Path(tmp) / "w.fxweights", FEATURES, seed=WEIGHT_SEED)
    net = fx.Net(wpath, P, max_batch=args.batch, precision="fp8", device=local)
    got = [None]
    if rank == 0:
        calib = np.stack([fx.synth_spiral((P, P, P), CALIB_SEED0 + i, fx.SPIRAL_CONFIG3) for i in range(4)])
        net.calibrate(calib)
        d_cal, _ = net.calibrate_schedule(calib, min_dice=SCHED_DICE)
        got = [(net.act_scales().tolist(), [l["precision"] for l in net.layers()], d_cal)]
    if world > 1:
        torch.distributed.broadcast_object_list(got, src=0)
        if rank != 0:
            net.set_act_scales(got[0][0])
            net.set_layer_precision(["fp8" if q == "fp8" else "f16" for q in got[0][1]])
    d_cal = got[0][2]
    rows = args.stream_rows or None
    sr = StreamRank(net, STREAM_SHAPE, ov, args.batch, rank=rank, world=world, group=group, rows=rows)
    z_lo, z_hi = sr.input_planes
    host_in = torch.empty((z_hi - z_lo, dy, dx), dtype=torch.uint8).pin_memory()
    fx.synth_spiral(STREAM_SHAPE, STREAM_SEED, fx.SPIRAL_CONFIG5, z_lo, z_hi, chunked=True, out=host_in.numpy())
    hin = host_in.numpy()
    host_out = torch.empty((4 * 64, dy, dx), dtype=torch.uint8).pin_memory()
    # warm-up: forwards of 8 tiles of this rank's input
    tiles = torch.from_numpy(np.ascontiguousarray(hin[:P, :P, :P])).cuda().repeat(args.batch, 1, 1)
    prob = torch.empty((args.batch, P, P, P), dtype=torch.float32, device="cuda")
    for _ in range(args.warmup):
        net.forward_dev(tiles.data_ptr(), args.batch, prob.data_ptr())
    torch.cuda.synchronize()
    del tiles, prob
    clocks = ClockSampler(local)
    clocks.start()
    l0 = fx.kernel_launches()
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    sr.run(lambda a, b: hin[a - z_lo:b - z_lo], out=host_out.numpy())
    secs = time.perf_counter() - t0
    launches = fx.kernel_launches() - l0
    clk = clocks.stop()
    fx.check(fx.lib().fx_net_device_status(net.handle))
    tot = np.array([sr.finalised, launches, (z_hi - z_lo) * dy * dx], dtype=np.float64)
    if world > 1:
        t = torch.tensor(tot)
        torch.distributed.all_reduce(t)
        m = torch.tensor([secs], dtype=torch.float64)
        torch.distributed.all_reduce(m, op=torch.distributed.ReduceOp.MAX)
        tot, secs = t.numpy(), float(m.item())
    value = tot[0] / secs / 1e6
    if rank == 0:
        nrows = sr.rows
        print(json.dumps({
            "metric": STREAM_METRIC, "value": value, "unit": "Mvoxels/s", "n_gpus": world, "steps": 1,
            "warmup": args.warmup, "ms_per_step": secs * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "e4m3 + f16 (calibrated schedule)",
            "data": "synthetic: 2048x4096x4096 u8 spiral sheet (pitch 14, thickness 3, N(170,15)/N(40,10), blur 1), "
                    "noise keyed per 64^3 chunk, seed 4; random-init Kaiming weights (seed 1)",
            "config": {"workload": f"out-of-core streaming: tile rows [0, {nrows}) of the 21 x 42 x 42 grid of 192^3 "
                                   "tiles at overlap 0.5, one step = the whole run, rows split over the GPUs, "
                                   "boundary chunk rows finalised by the lower GPU after an NVLink (IPC) band add",
                       "volume": list(STREAM_SHAPE), "patch": P, "overlap": ov, "batch": args.batch,
                       "tile_rows": nrows, "tiles": nrows * 42 * 42, "parallelism": f"tile-row ranges x{world}",
                       "l2": "inputs larger than L2: 3.2 GB of input planes per tile row"},
            "precision_schedule": dict(precision_report(net, None), calibration_dice=d_cal),
            "e2e": {"value": value, "unit": "Mvoxels/s", "h2d_bytes_per_step": int(tot[2]),
                    "d2h_bytes_per_step": int(tot[0]),
                    "path": "fenix_b200.stream.StreamRank: fx_gaccum_predict_row from pinned host planes, "
                            "fx_gaccum_finalize_below to pinned host u8, band export / add over IPC"},
            "clocks": clk, "gpu_launches": int(tot[1]),
        }))
    sr.close()
    net.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="fenix", choices=["fenix", "reference"])
    ap.add_argument("--precision", default="fp8", choices=["fp8", "fp8-all", "f16", "bf16"])
    ap.add_argument("--size", type=int, default=1024)
    ap.add_argument("--patch", type=int, default=128)
    ap.add_argument("--overlap", type=float, default=0.5)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-fxvol", action="store_true")
    ap.add_argument("--stream-rows", type=int, default=0,
                    help="stream workload: run the first R tile rows of the grid (0: all 21)")
    ap.add_argument("--minimal", action="store_true",
                    help="warm-up and timed steps only (no e2e, parity, peaks, baselines): for profiler launch lists")
    ap.add_argument("--workload", default="surface", choices=["surface", "ink", "stream"],
                    help="surface: the 1024^3 sliding-window benchmark (default); ink: batches of layer stacks; "
                         "stream: the out-of-core 2048x4096x4096 run, a bounded sample of tile rows")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "ink":
        return run_ink_reference(args) if args.impl == "reference" else run_ink(args)
    if args.workload == "stream":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the streaming sample has no separate reference arm; "
                              "its per-tile reference time is the surface workload's (same net, CPU libtorch)"}))
            return 0
        return run_stream(args)
    if args.impl == "reference":
        return run_reference_arm(args)

    import torch

    import fenix_b200 as fx
    from fenix_b200.shard import ShardedPredictor
    from fenix_b200.weights import make_plain_unet

    rank, world, local = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # host plumbing only (barriers, the IPC hand-over, the timing reduction): no NCCL anywhere
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        group = dist.group.WORLD

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    S, P = args.size, args.patch
    shape = (S, S, S)
    tmp = tempfile.mkdtemp(prefix=f"fxbench{rank}_")
    wpath = make_plain_unet(Path(tmp) / "w.fxweights", FEATURES, seed=WEIGHT_SEED)
    fp8 = args.precision.startswith("fp8")
    net = fx.Net(wpath, P, max_batch=args.batch, precision="fp8" if fp8 else args.precision, device=local)
    sched = None
    if fp8:
        # rank 0 calibrates (scales and schedule) and hands the result to the others, so every slab
        # is computed by the same network
        got = [None]
        if rank == 0:
            calib = np.stack([fx.synth_spiral((P, P, P), CALIB_SEED0 + i, fx.SPIRAL_CONFIG3) for i in range(4)])
            net.calibrate(calib)
            if args.precision == "fp8":
                d_cal, m_cal = net.calibrate_schedule(calib, min_dice=SCHED_DICE)
                sched = {"calibration_dice": d_cal, "calibration_max_abs": m_cal, "target_dice": SCHED_DICE}
            got = [(net.act_scales().tolist(), [l["precision"] for l in net.layers()], sched)]
        if world > 1:
            torch.distributed.broadcast_object_list(got, src=0)
            if rank != 0:
                scales, precs, sched = got[0]
                net.set_act_scales(scales)
                net.set_layer_precision(["fp8" if p == "fp8" else "f16" for p in precs])
    sp = ShardedPredictor(net, shape, args.overlap, args.batch, rank=rank, world=world, group=group)
    me = sp.me
    # this rank's input slab, generated on the host (pinned), and its output planes
    host_slab = torch.from_numpy(fx.synth_spiral(shape, VOLUME_SEED, fx.SPIRAL_CONFIG3, me.z_lo, max(me.z_hi, me.z_lo + 1))
                                 if me.z_hi > me.z_lo else np.zeros((1, S, S), np.uint8)).pin_memory()
    host_out = torch.empty((max(me.own_hi - me.own_lo, 1), S, S), dtype=torch.uint8).pin_memory()
    sp.slab.copy_(host_slab)
    torch.cuda.synchronize()
    # a real (non-null) stream: every kernel of the step and both timing events go on it
    stream = torch.cuda.Stream(device=local)

    def timed(fn, k):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("fx_timed")  # lets a profiler select the timed launches (--nvtx-include)
        ev0.record(stream)
        for _ in range(k):
            fn()
        ev1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        barrier()
        ms = ev0.elapsed_time(ev1)
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    dev_step = lambda: sp.run(stream=stream)  # noqa: E731  inputs resident in HBM
    if world == 1:
        # the drop-in call: fx_predict_volume with host (pinned) input and u8 output buffers
        hv, hu = host_slab.numpy(), host_out.numpy()

        def e2e_step():
            import ctypes as C

            opts = fx.InferOpts(P, args.overlap, 1, 0, args.batch)
            fx.check(fx.lib().fx_predict_volume(net.handle, hv.ctypes.data_as(C.POINTER(C.c_uint8)), S, S, S,
                                                C.byref(opts), None, hu.ctypes.data_as(C.POINTER(C.c_uint8))))
        e2e_path = "fx_predict_volume (C ABI) with pinned host u8 input and u8 output"
    else:
        e2e_step = lambda: sp.run(host_slab=host_slab, host_out=host_out, stream=stream)  # noqa: E731
        e2e_path = ("fenix_b200.shard.ShardedPredictor over fx_predict_tiles_dev / fx_accum_add (neighbour bands read "
                    "over NVLink) / fx_accum_finalize with pinned host input slab and output planes")
    for _ in range(args.warmup):
        dev_step()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    l0 = fx.kernel_launches()
    ms = timed(dev_step, args.steps)
    launches = fx.kernel_launches() - l0
    clk = clocks.stop()
    if args.minimal:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": float(S) ** 3 * args.steps / (ms / 1e3) / 1e6,
                              "unit": "Mvoxels/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                              "ms_per_step": ms / args.steps, "minimal": True, "gpu_launches": launches,
                              "config": workload_config(args, len(fx.tile_starts(S, P, args.overlap)) ** 3, world)}))
        sp.close()
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        net.close()
        return 0
    for _ in range(1):
        e2e_step()
    ms_e2e = timed(e2e_step, args.steps)
    fxv = None
    if world == 1 and not args.no_fxvol:
        try:
            fxv = fxvol_measure(host_slab.numpy(), host_out.numpy(), tmp)
        except Exception as e:  # reported, never fatal for the inference number
            fxv = {"failed": str(e)}
    # one profiled pass: per-launch CUDA events around every conv launch (not in the timed region)
    net.profile(True)
    dev_step()
    net.profile(False)
    prof = net.profile_read()
    layer_table = layer_times(net, dev_step, float(len(fx.tile_starts(S, P, args.overlap)) ** 3))
    h2d, d2h = sp.h2d_bytes, sp.d2h_bytes
    if world > 1:
        t = torch.tensor([float(launches), float(h2d), float(d2h)], dtype=torch.float64)
        torch.distributed.all_reduce(t)
        launches, h2d, d2h = (int(v) for v in t.tolist())
    parity_ok = S == 1024 and P == 128 and args.overlap == 0.5 and PARITY_CASE.exists()
    parity = parity_check(fx, net, args.batch, "fp8" if fp8 else args.precision) if rank == 0 and parity_ok else None
    # the two ends of the precision trade-off on the same net, for context (one GPU, fewer steps):
    # every layer on e4m3, and every layer on f16
    others = None
    if world == 1 and args.precision == "fp8":
        others = {}
        keep = [l["precision"] for l in net.layers()]
        for tag, sch in (("fp8_all", "fp8"), ("f16", "f16")):
            net.set_layer_precision([sch] * len(keep))
            dev_step()
            k = max(1, min(2, args.steps))
            t_ms = timed(dev_step, k)
            others[tag] = {"value": vox_of(S) * k / (t_ms / 1e3) / 1e6, "unit": "Mvoxels/s", "steps": k,
                           "ms_per_step": t_ms / k, "precision_schedule": precision_report(net, None),
                           "parity": parity_check(fx, net, args.batch, "fp8" if tag == "fp8_all" else "f16")
                           if parity_ok else None}
        net.set_layer_precision(["fp8" if q == "fp8" else "f16" for q in keep])
    vox = float(S) ** 3
    value = vox * args.steps / (ms / 1e3) / 1e6
    e2e = vox * args.steps / (ms_e2e / 1e3) / 1e6
    bf16_burst, bf16_sus, hbm, peak_src = peaks()
    conv_tflops = prof["conv_flops"] / (prof["conv_ms"] / 1e3) / 1e12
    # the tensor bound of the step's conv work: the measured rate of our own MMA-loop kernel
    # (fx_tc_peak) for each operand type, burst (best of 10 x 50 ms) and sustained (one 4 s run,
    # SM clock sampled), the e4m3 and 16-bit FLOPs each at their rate. The conv launches are timed
    # inside a seconds-long step, so the sustained rate is the denominator.
    f8 = prof["fp8_flops"] / max(prof["conv_flops"], 1.0)
    tc = measure_tc_peaks(fx, local)

    def mixed(p8, p16):
        return 1.0 / (f8 / p8 + (1.0 - f8) / p16)

    peak = mixed(tc["e4m3"]["sustained"], tc["f16"]["sustained"])
    peak_burst = mixed(tc["e4m3"]["burst"], tc["f16"]["burst"])
    cpu = None
    if world == 1 and not args.no_cpu_baseline and (ROOT / "oracle" / "_ref" / "ref_infer").exists():
        try:
            ext = min(S, 2 * P)
            crop, o = ref_crop(S, ext)
            per_tile, thr, nt, secs = cpu_reference(wpath, crop, P, args.overlap)
            tiles = len(fx.tile_starts(S, P, args.overlap)) ** 3
            cpu = {"value": vox / (tiles * per_tile) / 1e6, "unit": "Mvoxels/s", "cores": thr, "kind": "reference",
                   "sample": (f"reference predict_surface_filled fp32 over the central {ext}^3 crop [{o}, {o + ext})^3 "
                              f"of the same volume ({nt} tiles of {P}^3 at overlap {args.overlap}, {secs:.2f} s, "
                              f"{ext ** 3 / secs / 1e6:.3f} Mvoxels/s of that crop's output); the value is the "
                              f"per-tile time projected over the full volume's {tiles} tiles")}
        except Exception as e:  # reported, never fatal for the GPU number
            cpu = {"value": None, "unit": "Mvoxels/s", "cores": None, "kind": "reference", "sample": f"failed: {e}"}
    if rank == 0:
        tiles = len(fx.tile_starts(S, P, args.overlap)) ** 3
        line = {
            "metric": METRIC, "value": value, "unit": "Mvoxels/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": {"fp8": "e4m3 + f16 (calibrated schedule)", "fp8-all": "e4m3", "f16": "f16", "bf16": "bf16"}[args.precision],
            "data": f"synthetic: {S}^3 u8 spiral sheet (pitch 16, thickness 3, N(170,15)/N(40,10), blur 1, N(0,8) "
                    "speckle, seed 2); random-init Kaiming weights (seed 1); fp8 scales calibrated on 4 seeded patches",
            "config": workload_config(args, tiles, world),
            "roofline": {
                "bound": "tensor", "achieved": conv_tflops, "peak": peak, "unit": "TFLOP/s", "frac": conv_tflops / peak,
                "traffic": {"fp8-all": CONV_DRAM_BYTES_PER_TILE, "fp8": CONV_DRAM_BYTES_PER_TILE_SCHED}.get(args.precision),
                "traffic_unit": "DRAM bytes per 128^3 tile over the 22 conv launches (ncu capture, 256^3 bench)",
                "algorithmic_flops_per_tile": 945.2e9,
                "kernel": "conv_tc_kernel (all 22 conv launches of one forward, summed)",
                "peak_source": (f"measured on this GPU with fx_tc_peak (own tcgen05 MMA-loop kernel): e4m3 and f16 "
                                f"sustained rates (4 s each), weighted by the step's e4m3 FLOP share {f8:.3f}: "
                                "FLOPs / (f8 / p_e4m3 + f16 / p_f16); the conv kernel is timed inside a seconds-long step"),
                "tc_peaks_measured": tc,
                "cublas_bf16_measured": {"burst": bf16_burst, "sustained": bf16_sus, "source": f"MEASURED_PEAKS.json ({peak_src})"},
                "peak_burst": peak_burst, "frac_burst": conv_tflops / peak_burst,
                "conv_ms_per_step": prof["conv_ms"], "conv_flops_per_step": prof["conv_flops"],
                "fp8_flop_share": prof["fp8_flops"] / max(prof["conv_flops"], 1.0),
                "conv_share_of_step": prof["conv_ms"] / (ms / args.steps),
                # the whole step against the same denominator: its conv FLOPs over its device time
                "frac_step": prof["conv_flops"] / (ms / args.steps / 1e3) / 1e12 / peak,
                "frac_nominal": conv_tflops / mixed(4500.0, 2250.0),
                "nominal": "4.5 PFLOP/s e4m3, 2.25 PFLOP/s 16-bit (dense)",
            },
            "precision_schedule": precision_report(net, sched),
            "conv_layers": layer_table,
            "parity": parity,
            "other_schedules": others,
            "e2e": {"value": e2e, "unit": "Mvoxels/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": e2e_path},
            "cpu_baseline": cpu,
            "fxvol": fxv,
            "clocks": clk,
            "gpu_launches": launches,
        }
        print(json.dumps(line))
    sp.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    net.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
