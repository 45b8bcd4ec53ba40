"""Per-layer e4m3 sensitivity of a UNet against the reference's probability map, and the accuracy
and speed of calibrated precision schedules: the table behind an fp8 net's precision schedule.

  python -m fenix_b200.sensitivity --case tests/golden/net128_cfg3.npz [--targets 0.995,0.993,0.99]

The case file is one of the reference fixtures (weights seed, volume recipe, the reference's full
map). For every conv layer alone on e4m3 operands (the others f16): max |dp|, mean |dp| and Dice
of the 0.5-thresholded masks against the reference; then, for each Dice target, the layers
fx_net_calibrate_schedule picks on the calibration patches, their share of the FLOPs, the
schedule's agreement with the reference and the device time of one pass over a 256^3 volume
(27 tiles, batch 8). Prints a markdown report.
"""
from __future__ import annotations

import argparse
import tempfile
import time
from pathlib import Path

import numpy as np

from . import SPIRAL_CONFIG3, Net, synth_spiral
from .weights import make_plain_unet

KEYS = ("pitch", "thickness", "sheet_mean", "sheet_sd", "bg_mean", "bg_sd", "blur_sigma", "speckle_sd")


def _metrics(prob, ref):
    e = np.abs(prob - ref)
    a, b = prob >= 0.5, ref >= 0.5
    s = int(a.sum() + b.sum())
    return float(e.max()), float(e.mean()), (1.0 if s == 0 else 2.0 * float((a & b).sum()) / s)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True)
    ap.add_argument("--targets", default="0.995,0.993,0.99,0.985,0.98")
    ap.add_argument("--calib-seed", type=int, default=1000)
    args = ap.parse_args(argv)
    g = np.load(args.case)
    feats = tuple(int(v) for v in g["features"])
    P, ov = int(g["patch"]), float(g["overlap"])
    sp = dict(zip(KEYS, (float(v) for v in g["spiral"])))
    full, org, shape = (tuple(int(v) for v in g[k]) for k in ("full_shape", "crop_origin", "shape"))
    slab = synth_spiral(full, int(g["volume_seed"]), sp, org[0], org[0] + shape[0])
    vol = np.ascontiguousarray(slab[:, org[1]:org[1] + shape[1], org[2]:org[2] + shape[2]])
    ref = g["prob_u16"].astype(np.float32) / np.float32(65535.0)
    cal = np.stack([synth_spiral((P, P, P), args.calib_seed + i, SPIRAL_CONFIG3) for i in range(4)])
    big = synth_spiral((256, 256, 256), int(g["volume_seed"]), sp)
    with tempfile.TemporaryDirectory() as td:
        w = make_plain_unet(Path(td) / "w.fxweights", feats, seed=int(g["weight_seed"]))
        net = Net(w, P, max_batch=8, precision="fp8")
        net.calibrate(cal)
        layers = net.layers()
        n = len(layers)
        tot = sum(l["flops"] for l in layers)
        elig = [i for i, l in enumerate(layers) if l["precision"] == "fp8"]

        def run(sched):
            net.set_layer_precision(sched)
            prob, _ = net.predict_volume(vol, overlap=ov, batch=8, want_u8=False)
            return _metrics(prob, ref)

        def pass_ms():
            for _ in range(2):
                net.predict_volume(big, overlap=0.5, batch=8, want_u8=False, want_prob=False)
            t0 = time.perf_counter()
            for _ in range(3):
                net.predict_volume(big, overlap=0.5, batch=8, want_u8=False, want_prob=False)
            return (time.perf_counter() - t0) / 3 * 1e3

        all16, all8 = ["f16"] * n, ["fp8"] * n
        print(f"# e4m3 sensitivity: {Path(args.case).name}\n")
        print(f"Net {'/'.join(map(str, feats))}, {P}^3 tiles, overlap {ov}, volume {shape}; reference = the "
              "reference's own CPU inference (libtorch fp32), every voxel. Activation scales calibrated on 4 "
              f"seeded {P}^3 patches (seeds {args.calib_seed}..{args.calib_seed + 3}).\n")
        print("| layer | GFLOP per tile | alone on e4m3: max abs | mean abs | Dice | all but it on e4m3: Dice |")
        print("|---|---|---|---|---|---|")
        for k in elig:
            s1 = list(all16)
            s1[k] = "fp8"
            a = run(s1)
            s2 = list(all8)
            s2[k] = "f16"
            b = run(s2)
            print(f"| {layers[k]['name']} | {layers[k]['flops'] / 1e9:.2f} | {a[0]:.3e} | {a[1]:.2e} | {a[2]:.5f} | "
                  f"{b[2]:.5f} |")
        print("\n| schedule | e4m3 layers | e4m3 FLOP share | max abs | mean abs | Dice | 256^3 pass ms |")
        print("|---|---|---|---|---|---|---|")
        for tag, sched in (("all f16", all16), ("all e4m3", all8)):
            m = run(sched)
            lay = net.layers()
            share = sum(l["flops"] for l in lay if l["precision"] == "fp8") / tot
            print(f"| {tag} | {sum(l['precision'] == 'fp8' for l in lay)} | {share:.3f} | {m[0]:.3e} | {m[1]:.2e} | "
                  f"{m[2]:.5f} | {pass_ms():.1f} |")
        for t in (float(v) for v in args.targets.split(",")):
            dc, mc = net.calibrate_schedule(cal, min_dice=t)
            lay = net.layers()
            f8 = [l["name"] for l in lay if l["precision"] == "fp8"]
            share = sum(l["flops"] for l in lay if l["precision"] == "fp8") / tot
            prob, _ = net.predict_volume(vol, overlap=ov, batch=8, want_u8=False)
            m = _metrics(prob, ref)
            print(f"| calibrated, Dice target {t} (calibration {dc:.4f}) | {len(f8)}: {', '.join(f8)} | {share:.3f} | "
                  f"{m[0]:.3e} | {m[1]:.2e} | {m[2]:.5f} | {pass_ms():.1f} |")
        net.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
