"""Regenerate the golden fixtures in tests/golden/ from the REFERENCE's own code.

Runs only where the reference tree is present (it compiles oracle/_ref from it):
  * tiling_ref.npz  — tile starts, gaussian1d windows and accumulated weight profiles printed by
                      oracle/_ref/ref_tiler_dump (the reference's src/ml/tiling.hpp and
                      src/ml/global_accum.hpp), bit patterns kept exactly.
  * net_<case>.npz  — the reference's CPU inference (oracle/_ref/ref_infer: predict_surface_filled
                      + nets::ConvStack through libtorch, fp32, batch 2 so no fp16 round trip) on
                      seeded synthetic volumes with seeded random-init plain UNets: the u8-encoded
                      probability map, exact f32 values at 4096 sampled voxels, and sum / mean.
  * net128_<case>.npz — the benchmark configurations at their own 128^3 tile size, with the FULL
                      probability map (quantised to u16: round(p * 65535), error <= 7.7e-6):
                      config 1 (one 128^3 tile, 16/32/64/128 net, weight seed 0), config 2 (two
                      128^3 patches in one batch of 2, 32..320 net, weight seed 1, volume seed 1) and
                      config 3 (the central 192^3 crop [416, 608)^3 of the 1024^3 seed-2 speckled
                      volume: 8 tiles at overlap 0.5, so the middle third of every axis is a
                      blend of two tiles; the benchmark's weight seed 1).
  * feat_<case>.npz — InferOptions features through the reference's own predict_surface_filled on small
                      volumes (full maps as u16): octahedral TTA (tta_infer_dev), pct_minmax and
                      unit255 normalisation (norm_patch), the output core crop, the constant-input
                      tile filter of predict-scroll, and a one-class sigmoid head.
  * resenc_<case>.npz — the same with the reference's own nets::ResEncUNet (residual encoder,
                      optional scSE, plain or task naming) loaded from seeded random-init weights.
  * resenc_ink.npz — the reference's predict-ink configuration (src/ml/inference.cpp:898-908): its
                      nets::ResEncUNet with a task head (shared_encoder + shared_decoder +
                      task_heads.ink, no scSE, one class), sigmoid and pct_minmax normalisation,
                      through its own predict_surface_filled on a papyrus layer stack; full map u16.
  * ink_<case>.npz — the layer-stack (wide-ink) net: 64/128/256/512 features, stride (1, 2, 2) at
                      stages 1-2 and (2, 2, 2) at stage 3, one class + sigmoid, anisotropic tiles.
                      The reference's nets take one int stride per stage and its window tiles cubes,
                      so this map comes from the C ORACLE (fxo_predict_tiled), whose cube path the
                      net_* / net128_* fixtures pin against the reference and whose anisotropic
                      forward tests/test_ink_oracle.py checks against PyTorch fp32. Full map as u16.
  * ckpt_ref.npz   — a checkpoint file written by the reference itself: predict_surface_filled with
                      ckpt_path set, its filler failing after 3 patches so that it saves its
                      progress (src/ml/infer.hpp:840-846), as raw bytes; and the same run's full map
                      uninterrupted (u16). The GPU path must resume the reference's file.
  * hash64.npz     — the reference's own hash64 (src/core/hash.hpp via oracle/_ref/ref_hash) of
                      fixed byte strings and a chained 1 MiB stream: the identity hashes of its
                      prediction checkpoints.
  * fxvol_tiles.npz — the reference's encode_tile_dct payloads of the 64^3 chunks of
                      tests/golden/fxvol_cases.py, and SHA-256 digests of its decode_tile_dct output
                      (u8, and the f32 reconstruction) of those payloads (oracle/_ref/ref_fxvol).
  * fxvol_small.fxvol + fxvol_small.npz — an archive written by the reference's
                      VolumeArchive::create + write_volume<u8> + close from the fixture volume, the
                      coverage of every chunk of every LOD, and the digest of read_volume_as<u8>(0).

usage: python tests/golden/make_golden.py [--only CASE]
"""
from __future__ import annotations

import argparse
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

import fenix_b200 as fx  # noqa: E402
from fenix_b200.weights import make_plain_unet, make_resenc_unet  # noqa: E402
from oracle import oracle as orc  # noqa: E402

# name: (features, weight seed, volume shape, volume seed, spiral params, patch, overlap)
CASES = {
    "small3": ((16, 32, 64), 5, (72, 64, 80), 7, fx.SPIRAL_CONFIG1, 64, 0.5),
    "cfg1_p64": ((16, 32, 64, 128), 0, (64, 96, 64), 11, fx.SPIRAL_CONFIG1, 64, 0.25),
    "cfg2_p64": ((32, 64, 128, 256, 320), 1, (64, 64, 64), 1, fx.SPIRAL_CONFIG1, 64, 0.5),
    "cfg3_p64": ((32, 64, 128, 256, 320), 2, (96, 96, 96), 2, fx.SPIRAL_CONFIG3, 64, 0.5),
}

# name: (features, weight seed, full volume shape, crop origin (None: whole), crop extent, volume
# seed, spiral params, patch, overlap)
CASES128 = {
    "cfg1": ((16, 32, 64, 128), 0, (128, 128, 128), None, None, 0, fx.SPIRAL_CONFIG1, 128, 0.5),
    "cfg2": ((32, 64, 128, 256, 320), 1, (256, 128, 128), None, None, 1, fx.SPIRAL_CONFIG1, 128, 0.0),
    "cfg3": ((32, 64, 128, 256, 320), 1, (1024, 1024, 1024), (416, 416, 416), (192, 192, 192), 2, fx.SPIRAL_CONFIG3,
             128, 0.5),
}


def volume128(name):
    """The input volume of a net128 case (a crop of the full synthetic where the case has one)."""
    feats, wseed, full, org, ext, vseed, sp, P, ov = CASES128[name]
    if org is None:
        return fx.synth_spiral(full, vseed, sp)
    slab = fx.synth_spiral(full, vseed, sp, org[0], org[0] + ext[0])
    return np.ascontiguousarray(slab[:, org[1]:org[1] + ext[1], org[2]:org[2] + ext[2]])


# name: (features, ncls, weight seed, volume shape, volume seed, patch, overlap, reference options)
FEATS = {
    "tta8": ((16, 32, 64, 128), 2, 3, (96, 80, 72), 21, 64, 0.5, {"tta": 8}),
    "tta48": ((16, 32, 64), 2, 4, (64, 64, 64), 22, 64, 0.5, {"tta": 48}),
    "pct": ((16, 32, 64, 128), 2, 5, (96, 80, 72), 23, 64, 0.5, {"norm": "pct_minmax"}),
    "unit255": ((16, 32, 64, 128), 2, 6, (96, 80, 72), 24, 64, 0.5, {"norm": "unit255"}),
    "core": ((16, 32, 64, 128), 2, 7, (96, 80, 72), 25, 64, 0.5, {"core": (16, 8, 4, 48, 40, 44)}),
    "skipconst": ((16, 32, 64, 128), 2, 8, (128, 64, 96), 26, 64, 0.5, {"skipconst": 1}),
    "sigmoid": ((16, 32, 64, 128), 1, 9, (96, 80, 72), 27, 64, 0.5, {"sigmoid": 1}),
}


def feat_volume(name):
    """The input volume of a feat case: the spiral synthetic (planes [0, 72) held at one value for
    the constant-tile case)."""
    feats, ncls, wseed, shape, vseed, P, ov, ropt = FEATS[name]
    vol = fx.synth_spiral(shape, vseed, fx.SPIRAL_CONFIG1)
    if name == "skipconst":
        vol[:72] = 40
    return vol


# name: (weight seed, stack shape, papyrus seed, stack index, tile (z, y, x), overlap)
INK = {
    "small": (3, (24, 112, 112), 3, 0, (16, 64, 64), 0.25),
}


def ink_case(name):
    from fenix_b200.weights import INK_FEATURES, INK_STRIDES
    from oracle import netgen

    wseed, shape, vseed, stack, tile, ov = INK[name]
    vol = orc.synth_papyrus(shape, vseed, stack)
    with tempfile.TemporaryDirectory() as td:
        w = netgen.make_plain_unet(Path(td) / "w.fxweights", INK_FEATURES, ncls=1, seed=wseed, strides=INK_STRIDES)
        prob = orc.Net(w).predict_tiled(vol, tile, ov, channel=0, sigmoid=1)
    np.savez_compressed(HERE / f"ink_{name}.npz", features=np.array(INK_FEATURES), strides=np.array(INK_STRIDES),
                        weight_seed=wseed, shape=np.array(shape), volume_seed=vseed, stack=stack, tile=np.array(tile),
                        overlap=ov, prob_u16=np.round(prob.astype(np.float64) * 65535.0).astype(np.uint16),
                        source="oracle")
    print(f"ink_{name}: mean {prob.mean():.4f}, > 0.5: {(prob > 0.5).mean():.3f}")


# name: (features, blocks, scSE, plain naming, weight seed, volume shape, volume seed, patch, overlap)
RESENC = {
    "plain": ((16, 32, 64, 64), (1, 2, 2, 1), False, True, 6, (80, 72, 96), 8, 64, 0.5),
    "scse": ((16, 32, 64), (1, 2, 2), True, False, 7, (64, 80, 64), 9, 64, 0.5),
}


def tiling():
    out = subprocess.run([str(orc.REF / "ref_tiler_dump")], capture_output=True, text=True, check=True).stdout
    d = {}
    for line in out.splitlines():
        head, vals = line.split(":", 1)
        parts = head.split()
        kind = parts[0]
        key = "_".join(parts[1:])
        vals = vals.split()
        if kind == "starts":
            d[f"starts_{key}"] = np.array([int(v) for v in vals], dtype=np.int64)
        else:
            d[f"{kind}_{key}"] = np.array([float.fromhex(v) for v in vals], dtype=np.float32)
    np.savez_compressed(HERE / "tiling_ref.npz", **d)
    print(f"tiling_ref.npz: {len(d)} arrays")


def net_case(name):
    feats, wseed, shape, vseed, sp, P, ov = CASES[name]
    with tempfile.TemporaryDirectory() as td:
        w = make_plain_unet(Path(td) / "w.fxweights", feats, nconv=2, ncls=2, seed=wseed)
        vol = fx.synth_spiral(shape, vseed, sp)
        prob, info = orc.ref_infer(w, vol, P, ov, batch=2)
    rng = np.random.default_rng(1234)
    idx = rng.choice(prob.size, size=min(4096, prob.size), replace=False).astype(np.int64)
    np.savez_compressed(
        HERE / f"net_{name}.npz",
        u8=orc.prob_to_u8(prob),
        sample_idx=idx,
        sample_val=prob.reshape(-1)[idx],
        prob_sum=np.float64(prob.astype(np.float64).sum()),
        features=np.array(feats, dtype=np.int64),
        weight_seed=np.int64(wseed),
        shape=np.array(shape, dtype=np.int64),
        volume_seed=np.int64(vseed),
        spiral=np.array([sp[k] for k in ("pitch", "thickness", "sheet_mean", "sheet_sd", "bg_mean", "bg_sd",
                                         "blur_sigma", "speckle_sd")]),
        patch=np.int64(P),
        overlap=np.float64(ov),
        ref_seconds=np.float64(info["seconds"]),
        ref_threads=np.int64(info["threads"]),
    )
    print(f"net_{name}.npz: shape {shape}, {info}")


def net128_case(name):
    feats, wseed, full, org, ext, vseed, sp, P, ov = CASES128[name]
    vol = volume128(name)
    with tempfile.TemporaryDirectory() as td:
        w = make_plain_unet(Path(td) / "w.fxweights", feats, nconv=2, ncls=2, seed=wseed)
        prob, info = orc.ref_infer(w, vol, P, ov, batch=2)
    np.savez_compressed(
        HERE / f"net128_{name}.npz",
        prob_u16=np.round(np.clip(prob, 0.0, 1.0).astype(np.float64) * 65535.0).astype(np.uint16),
        prob_sum=np.float64(prob.astype(np.float64).sum()),
        features=np.array(feats, dtype=np.int64),
        weight_seed=np.int64(wseed),
        full_shape=np.array(full, dtype=np.int64),
        crop_origin=np.array(org if org else (0, 0, 0), dtype=np.int64),
        shape=np.array(vol.shape, dtype=np.int64),
        volume_seed=np.int64(vseed),
        spiral=np.array([sp[k] for k in ("pitch", "thickness", "sheet_mean", "sheet_sd", "bg_mean", "bg_sd",
                                         "blur_sigma", "speckle_sd")]),
        patch=np.int64(P),
        overlap=np.float64(ov),
        ref_seconds=np.float64(info["seconds"]),
        ref_threads=np.int64(info["threads"]),
    )
    print(f"net128_{name}.npz: shape {vol.shape}, {info}")


def feat_case(name):
    feats, ncls, wseed, shape, vseed, P, ov, ropt = FEATS[name]
    vol = feat_volume(name)
    with tempfile.TemporaryDirectory() as td:
        w = make_plain_unet(Path(td) / "w.fxweights", feats, nconv=2, ncls=ncls, seed=wseed)
        prob, info = orc.ref_infer(w, vol, P, ov, batch=2, **ropt)
    np.savez_compressed(
        HERE / f"feat_{name}.npz",
        prob_u16=np.round(np.clip(prob, 0.0, 1.0).astype(np.float64) * 65535.0).astype(np.uint16),
        features=np.array(feats, dtype=np.int64), ncls=np.int64(ncls), weight_seed=np.int64(wseed),
        shape=np.array(shape, dtype=np.int64), volume_seed=np.int64(vseed), patch=np.int64(P),
        overlap=np.float64(ov), options=np.array(repr(ropt)),
    )
    print(f"feat_{name}.npz: {prob.shape}, {info}")


def resenc_case(name):
    feats, blocks, se, plain, wseed, shape, vseed, P, ov = RESENC[name]
    sp = fx.SPIRAL_CONFIG1
    with tempfile.TemporaryDirectory() as td:
        w = make_resenc_unet(Path(td) / "w.fxweights", feats, blocks, ncls=2, se=se, plain_naming=plain, seed=wseed)
        vol = fx.synth_spiral(shape, vseed, sp)
        prob, info = orc.ref_infer(w, vol, P, ov, batch=2)
    rng = np.random.default_rng(4321)
    idx = rng.choice(prob.size, size=min(4096, prob.size), replace=False).astype(np.int64)
    np.savez_compressed(
        HERE / f"resenc_{name}.npz",
        u8=orc.prob_to_u8(prob),
        sample_idx=idx,
        sample_val=prob.reshape(-1)[idx],
        features=np.array(feats, dtype=np.int64),
        blocks=np.array(blocks, dtype=np.int64),
        se=np.int64(se),
        plain_naming=np.int64(plain),
        weight_seed=np.int64(wseed),
        shape=np.array(shape, dtype=np.int64),
        volume_seed=np.int64(vseed),
        patch=np.int64(P),
        overlap=np.float64(ov),
    )
    print(f"resenc_{name}.npz: shape {shape}, {info}")


def fxvol():
    import hashlib
    import os

    sys.path.insert(0, str(HERE))
    import fxvol_cases as fc

    tool = str(orc.REF / "ref_fxvol")
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    d = {}
    with tempfile.TemporaryDirectory() as td:
        for dtype, cases, gen in (("u8", fc.TILE_CASES_U8, fc.chunk_u8), ("f32", fc.TILE_CASES_F32, fc.chunk_f32)):
            for k, (kind, q) in enumerate(cases):
                src = Path(td) / "in.raw"
                gen(kind).tofile(src)
                subprocess.run([tool, "enc", dtype, repr(q), "1", str(src), f"{td}/p.bin"], check=True)
                blob = (Path(td) / "p.bin").read_bytes()
                n = int.from_bytes(blob[:4], "little")
                key = f"{dtype}_{kind}_q{q:g}"
                d[f"pay_{key}"] = np.frombuffer(blob[4:4 + n], dtype=np.uint8)
                subprocess.run([tool, "dec", "u8", repr(q), f"{td}/p.bin", f"{td}/o.raw"], check=True)
                d[f"sha_u8_{key}"] = np.array(sha(np.fromfile(f"{td}/o.raw", dtype=np.uint8)))
                subprocess.run([tool, "dec", "f32", repr(q), f"{td}/p.bin", f"{td}/o.raw"], check=True)
                d[f"sha_f32_{key}"] = np.array(sha(np.fromfile(f"{td}/o.raw", dtype=np.float32)))
        np.savez_compressed(HERE / "fxvol_tiles.npz", **d)
        vol = fc.archive_volume()
        vol.tofile(f"{td}/v.raw")
        dz, dy, dx = fc.ARCHIVE_DIMS
        out = HERE / "fxvol_small.fxvol"
        if out.exists():
            os.remove(out)
        subprocess.run([tool, "write", repr(fc.ARCHIVE_Q), str(dz), str(dy), str(dx), f"{td}/v.raw", str(out)], check=True)
        subprocess.run([tool, "read", str(out), f"{td}/r.raw"], check=True, capture_output=True)
        slots = subprocess.run([tool, "slots", str(out)], check=True, capture_output=True, text=True).stdout
        cov = np.array([[int(v) for v in line.split()] for line in slots.splitlines()], dtype=np.int64)
        np.savez_compressed(HERE / "fxvol_small.npz", coverage=cov,
                            sha_read=np.array(sha(np.fromfile(f"{td}/r.raw", dtype=np.uint8))))
    print(f"fxvol: {len(fc.TILE_CASES_U8) + len(fc.TILE_CASES_F32)} tiles, archive {out.stat().st_size} bytes")


CKPT = dict(features=(16, 32, 64, 128), weight_seed=0, shape=(96, 64, 128), volume_seed=13, patch=64, overlap=0.5,
            batch=2, stop_after=3, whash=11, ihash=22)


INK_RESENC = dict(features=(16, 32, 64), blocks=(1, 2, 2), weight_seed=12, shape=(64, 96, 112), volume_seed=3,
                  stack=4, patch=64, overlap=0.25)


def resenc_ink():
    c = INK_RESENC
    vol = orc.synth_papyrus(c["shape"], c["volume_seed"], c["stack"])
    with tempfile.TemporaryDirectory() as td:
        w = make_resenc_unet(Path(td) / "w.fxweights", c["features"], c["blocks"], ncls=1, se=False, plain_naming=False,
                             seed=c["weight_seed"], task="ink", task_head=True)
        prob, info = orc.ref_infer(w, vol, c["patch"], c["overlap"], batch=2, sigmoid=1, channel=0, norm="pct_minmax")
    np.savez_compressed(HERE / "resenc_ink.npz", prob_u16=np.round(prob.astype(np.float64) * 65535.0).astype(np.uint16),
                        **{k: np.array(v) for k, v in c.items()})
    print(f"resenc_ink: mean {prob.mean():.4f}, > 0.5: {(prob > 0.5).mean():.3f}")


def ckpt_ref():
    c = CKPT
    vol = fx.synth_spiral(c["shape"], c["volume_seed"], fx.SPIRAL_CONFIG1)
    with tempfile.TemporaryDirectory() as td:
        w = make_plain_unet(Path(td) / "w.fxweights", c["features"], seed=c["weight_seed"])
        ck = Path(td) / "run.ckpt"
        try:
            orc.ref_infer(w, vol, c["patch"], c["overlap"], batch=c["batch"], ckpt=str(ck), whash=c["whash"],
                          ihash=c["ihash"], stopafter=c["stop_after"])
            raise RuntimeError("ckpt_ref: the interrupted reference run did not fail")
        except subprocess.CalledProcessError:
            pass
        raw = ck.read_bytes()
        full, _ = orc.ref_infer(w, vol, c["patch"], c["overlap"], batch=c["batch"])
    done = int.from_bytes(raw[48:56], "little")
    np.savez_compressed(HERE / "ckpt_ref.npz", ckpt=np.frombuffer(raw, dtype=np.uint8),
                        prob_u16=np.round(full.astype(np.float64) * 65535.0).astype(np.uint16),
                        **{k: np.array(v) for k, v in c.items()})
    print(f"ckpt_ref: {len(raw)} bytes, {done} tiles done")


def hash64():
    out = subprocess.run([str(orc.REF / "ref_hash")], capture_output=True, text=True, check=True).stdout
    rows, chain = [], None
    for line in out.splitlines():
        f = line.split()
        if f[0] == "bytes":
            rows.append((int(f[1]), int(f[2]), int(f[3])))
        elif f[0] == "chain":
            chain = int(f[1])
    a = np.array(rows, dtype=np.uint64)
    np.savez_compressed(HERE / "hash64.npz", lens=a[:, 0], h0=a[:, 1], hseed=a[:, 2], chain=np.uint64(chain))
    print(f"hash64: {len(rows)} strings + chain")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "all", "ref"], check=True)
    if a.only in (None, "tiling"):
        tiling()
    for name in CASES:
        if a.only in (None, name):
            net_case(name)
    for name in CASES128:
        if a.only in (None, "net128_" + name):
            net128_case(name)
    for name in FEATS:
        if a.only in (None, "feat_" + name):
            feat_case(name)
    for name in RESENC:
        if a.only in (None, "resenc_" + name):
            resenc_case(name)
    for name in INK:
        if a.only in (None, "ink_" + name):
            ink_case(name)
    if a.only in (None, "hash64"):
        hash64()
    if a.only in (None, "ckpt_ref"):
        ckpt_ref()
    if a.only in (None, "resenc_ink"):
        resenc_ink()
    if a.only in (None, "fxvol"):
        fxvol()


if __name__ == "__main__":
    main()
