/* synth.c — the spiral-sheet synthetic CT of the benchmark configurations, generated on the
 * checker side. TEST INFRASTRUCTURE ONLY: it lets the reference arm of the benchmark and the
 * golden-fixture scripts make the workload's input volume without loading the product library.
 * Its bytes equal fx_synth_spiral's (include/fenix_b200_synth.h), which a CPU test checks.
 *
 * The recipe (the benchmark's synthetic-input description): an Archimedean spiral r = b phi,
 * b = pitch / (2 pi), centred in the (y, x) plane and extruded along z; a voxel is sheet when its
 * radial distance to the nearest turn is below thickness / 2. Intensity N(sheet_mean, sheet_sd) on
 * the sheet and N(bg_mean, bg_sd) elsewhere (Box-Muller over PCG-XSH-RR 64/32, O'Neill 2014, one
 * stream per (z, y) row), a separable Gaussian blur (radius ceil(3 sigma), edge clamp), then
 * N(0, speckle_sd) speckle from a second per-row stream, clip to [0, 255], round half up. */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifndef M_PI
#define M_PI 3.14159265358979323846
#endif

typedef struct fxo_spiral {
    double pitch, thickness, sheet_mean, sheet_sd, bg_mean, bg_sd, blur_sigma, speckle_sd;
} fxo_spiral;

typedef struct {
    uint64_t state, inc;
} pcg_t;

static uint32_t pcg_next(pcg_t* r) {
    const uint64_t old = r->state;
    r->state = old * 6364136223846793005ULL + r->inc;
    const uint32_t xs = (uint32_t)(((old >> 18u) ^ old) >> 27u);
    const uint32_t rot = (uint32_t)(old >> 59u);
    return (xs >> rot) | (xs << ((~rot + 1u) & 31u));
}

static pcg_t pcg_seed(uint64_t seed, uint64_t stream) {
    pcg_t r;
    r.inc = (stream << 1u) | 1u;
    r.state = 0;
    pcg_next(&r);
    r.state += seed;
    pcg_next(&r);
    return r;
}

static float pcg_uniform(pcg_t* r) { return (float)(pcg_next(r) >> 8) * (1.0f / 16777216.0f); }

static float pcg_normal(pcg_t* r) {
    float u1 = pcg_uniform(r);
    if (u1 < 1e-7f) u1 = 1e-7f;
    const float u2 = pcg_uniform(r);
    return sqrtf(-2.0f * logf(u1)) * cosf(6.28318530718f * u2);
}

static float sheet_dist(double y, double x, double cy, double cx, double pitch) {
    const double ry = y - cy, rx = x - cx;
    const double r = sqrt(ry * ry + rx * rx);
    const double th = atan2(ry, rx) + M_PI;
    const double b = pitch / (2.0 * M_PI);
    double k = round((r / b - th) / (2.0 * M_PI));
    if (k < 0) k = 0;
    return (float)fabs(r - b * (th + 2.0 * M_PI * k));
}

static int64_t clampi(int64_t v, int64_t lo, int64_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* out: [z_end - z_begin][dy][dx]; 0 on success */
int fxo_synth_spiral(uint8_t* out, int64_t dz, int64_t dy, int64_t dx, const fxo_spiral* p, uint64_t seed,
                     int64_t z_begin, int64_t z_end) {
    if (!out || !p || dz < 1 || dy < 1 || dx < 1 || z_begin < 0 || z_end > dz || z_begin >= z_end) return 1;
    const double cy = (dy - 1) / 2.0, cx = (dx - 1) / 2.0;
    const int rad = p->blur_sigma > 0 ? (int)ceil(3.0 * p->blur_sigma) : 0;
    float k[64];
    if (rad > 31) return 1;
    for (int i = 0; i < 2 * rad + 1; ++i) k[i] = 1.f;
    if (rad) {
        double s = 0;
        for (int i = -rad; i <= rad; ++i) s += exp(-0.5 * i * i / (p->blur_sigma * p->blur_sigma));
        for (int i = -rad; i <= rad; ++i) k[i + rad] = (float)(exp(-0.5 * i * i / (p->blur_sigma * p->blur_sigma)) / s);
    }
    const int64_t plane = dy * dx;
    uint8_t* sheet = malloc((size_t)plane);
    if (!sheet) return 1;
#pragma omp parallel for schedule(static)
    for (int64_t y = 0; y < dy; ++y)
        for (int64_t x = 0; x < dx; ++x)
            sheet[y * dx + x] = sheet_dist((double)y, (double)x, cy, cx, p->pitch) < 0.5 * p->thickness ? 1 : 0;
    int rc = 0;
    const int64_t chunk = 32;
    for (int64_t c0 = z_begin; c0 < z_end && !rc; c0 += chunk) {
        const int64_t c1 = c0 + chunk < z_end ? c0 + chunk : z_end;
        const int64_t g0 = c0 - rad > 0 ? c0 - rad : 0, g1 = c1 + rad < dz ? c1 + rad : dz;
        const int64_t ng = g1 - g0;
        float* a = malloc(sizeof(float) * (size_t)(ng * plane));
        float* tmps = rad ? malloc(sizeof(float) * (size_t)(ng * plane)) : NULL;
        if (!a || (rad && !tmps)) {
            free(a);
            free(tmps);
            rc = 1;
            break;
        }
#pragma omp parallel for schedule(static)
        for (int64_t zi = 0; zi < ng; ++zi) {
            const int64_t z = g0 + zi;
            float* q = a + zi * plane;
            for (int64_t y = 0; y < dy; ++y) {
                pcg_t r = pcg_seed(seed, (uint64_t)(z * dy + y) + 0x9E3779B97F4A7C15ull);
                for (int64_t x = 0; x < dx; ++x) {
                    const float n = pcg_normal(&r);
                    q[y * dx + x] = sheet[y * dx + x] ? (float)(p->sheet_mean + p->sheet_sd * n)
                                                      : (float)(p->bg_mean + p->bg_sd * n);
                }
            }
            if (!rad) continue;
            float* tmp = tmps + zi * plane;
            for (int64_t y = 0; y < dy; ++y)
                for (int64_t x = 0; x < dx; ++x) {
                    float s = 0.f;
                    for (int i = -rad; i <= rad; ++i) s += k[i + rad] * q[y * dx + clampi(x + i, 0, dx - 1)];
                    tmp[y * dx + x] = s;
                }
            for (int64_t y = 0; y < dy; ++y)
                for (int64_t x = 0; x < dx; ++x) {
                    float s = 0.f;
                    for (int i = -rad; i <= rad; ++i) s += k[i + rad] * tmp[clampi(y + i, 0, dy - 1) * dx + x];
                    q[y * dx + x] = s;
                }
        }
#pragma omp parallel for schedule(static)
        for (int64_t zo = 0; zo < c1 - c0; ++zo) {
            const int64_t z = c0 + zo;
            uint8_t* o = out + (z - z_begin) * plane;
            for (int64_t y = 0; y < dy; ++y) {
                pcg_t r = pcg_seed(seed ^ 0xA5A5A5A5DEADBEEFull, (uint64_t)(z * dy + y) + 0x632BE59BD9B4E019ull);
                for (int64_t x = 0; x < dx; ++x) {
                    float s;
                    if (rad) {
                        s = 0.f;
                        for (int i = -rad; i <= rad; ++i) {
                            const int64_t zz = clampi(z + i, 0, dz - 1);
                            s += k[i + rad] * a[(zz - g0) * plane + y * dx + x];
                        }
                    } else {
                        s = a[(z - g0) * plane + y * dx + x];
                    }
                    if (p->speckle_sd > 0) s += (float)p->speckle_sd * pcg_normal(&r);
                    s = fminf(255.f, fmaxf(0.f, s));
                    o[y * dx + x] = (uint8_t)floorf(s + 0.5f);
                }
            }
        }
        free(a);
        free(tmps);
    }
    free(sheet);
    return rc;
}
