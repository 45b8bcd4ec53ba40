/* fenix_b200_synth.h — deterministic synthetic CT volumes for parity tests and benchmarks (not
 * part of the inference path): an Archimedean spiral sheet extruded along z.
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

#ifdef __cplusplus
}
#endif

#endif
