/* fenix_b200_synth.h — deterministic synthetic CT volumes for parity tests and benchmarks (not
 * part of the inference path): an Archimedean spiral sheet extruded along z (fx_synth_spiral),
 * and papyrus layer stacks with ink (fx_synth_papyrus, below).
 *
 * A voxel is "sheet" when its radial distance to the nearest turn of r = pitch * phi / (2 pi)
 * (centred in the (y, x) plane) is below thickness / 2. Intensity: N(sheet_mean, sheet_sd) on
 * the sheet, N(bg_mean, bg_sd) elsewhere, then a separable Gaussian blur (sigma blur_sigma,
 * radius ceil(3 sigma), edge clamp), then N(0, speckle_sd) speckle, clip to [0, 255], round.
 * Noise comes from PCG32 streams keyed by each (z, y) row, so any z-range [z_begin, z_end)
 * regenerates exactly the bytes of the whole volume. Returns 0 on success. */
#ifndef FENIX_B200_SYNTH_H
#define FENIX_B200_SYNTH_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct fx_spiral_params {
    double pitch;      /* voxels between successive turns */
    double thickness;  /* sheet thickness in voxels */
    double sheet_mean, sheet_sd;
    double bg_mean, bg_sd;
    double blur_sigma; /* 0 = no blur */
    double speckle_sd; /* 0 = no speckle */
} fx_spiral_params;

/* out: [z_end - z_begin][dy][dx] */
int fx_synth_spiral(uint8_t* out, int64_t dz, int64_t dy, int64_t dx, const fx_spiral_params* params, uint64_t seed,
                    int64_t z_begin, int64_t z_end);
/* The same recipe with the noise keyed per 64^3 chunk (the out-of-core workload's volume): the
 * normals of a 64-voxel run of row (z, y) inside chunk (z / 64, y / 64, x / 64) come from the PCG
 * stream ((chunk index << 12) | (z % 64) << 6 | (y % 64)), chunk index = (cz * ncy + cy) * ncx + cx,
 * so any chunk (with the blur's 3-voxel margin) regenerates from its own and its neighbours'
 * streams. Bytes differ from fx_synth_spiral's. */
int fx_synth_spiral_chunked(uint8_t* out, int64_t dz, int64_t dy, int64_t dx, const fx_spiral_params* params,
                            uint64_t seed, int64_t z_begin, int64_t z_end);

/* Papyrus layer stacks with ink, the layer-stack (wide-ink) workload's input: one surface-normal
 * layer stack [dz][dy][dx] (z = the layer axis) per call, number `stack` of a seeded series.
 *
 * Fibre texture: white N(0, 1) noise filtered by a separable Gaussian of sigma (sigma_z, sigma_y,
 * sigma_x) per axis (radius ceil(3 sigma), weights exp(-i^2 / 2 sigma^2) normalised, edge clamp,
 * passes along x, then y, then z), rescaled by sd / sqrt(sum kz^2 * sum ky^2 * sum kx^2) so its
 * standard deviation is sd, around `mean`. Ink: a second white-noise plane [dy][dx] filtered by a
 * 2D Gaussian of sigma ink_sigma; the floor(ink_fraction * dy * dx) columns with the largest
 * values (every column >= the k-th largest) are ink and get +ink_delta on every layer. Clip to
 * [0, 255], round half up. Noise streams: PCG32 keyed by the stack and the (z, y) row (texture)
 * or the y row (ink). `ink` (NULL = not wanted) receives the [dy][dx] 0/1 ink mask.
 * Returns 0 on success. */
typedef struct fx_papyrus_params {
    double sigma_z, sigma_y, sigma_x; /* fibre texture filter, voxels (0 = none along that axis) */
    double mean, sd;                  /* texture intensity */
    double ink_sigma;                 /* ink blob filter, voxels */
    double ink_fraction;              /* share of (y, x) columns carrying ink */
    double ink_delta;                 /* intensity added on ink */
} fx_papyrus_params;

int fx_synth_papyrus(uint8_t* out, uint8_t* ink, int64_t dz, int64_t dy, int64_t dx, const fx_papyrus_params* params,
                     uint64_t seed, int64_t stack);

#ifdef __cplusplus
}
#endif

#endif
