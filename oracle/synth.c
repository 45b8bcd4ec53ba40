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

/* The normals of row (z, y) into f[0, dx): one PCG stream per row, or (chunked) one per 64-voxel
 * run inside its 64^3 chunk, stream ((chunk << 12) | (z % 64) << 6 | (y % 64)) + salt. */
static void row_normals(uint64_t seed, uint64_t salt, int chunked, int64_t z, int64_t y, int64_t dy, int64_t dx,
                        float* f) {
    if (!chunked) {
        pcg_t r = pcg_seed(seed, (uint64_t)(z * dy + y) + salt);
        for (int64_t x = 0; x < dx; ++x) f[x] = pcg_normal(&r);
        return;
    }
    const int64_t ncy = (dy + 63) / 64, ncx = (dx + 63) / 64;
    for (int64_t x0 = 0; x0 < dx; x0 += 64) {
        const uint64_t chunk = (uint64_t)(((z >> 6) * ncy + (y >> 6)) * ncx + (x0 >> 6));
        pcg_t r = pcg_seed(seed, ((chunk << 12) | ((uint64_t)(z & 63) << 6) | (uint64_t)(y & 63)) + salt);
        for (int64_t x = x0; x < dx && x < x0 + 64; ++x) f[x] = pcg_normal(&r);
    }
}

static int synth_spiral_impl(uint8_t* out, int64_t dz, int64_t dy, int64_t dx, const fxo_spiral* p, uint64_t seed,
                             int64_t z_begin, int64_t z_end, int chunked) {
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
                row_normals(seed, 0x9E3779B97F4A7C15ull, chunked, z, y, dy, dx, q + y * dx);
                for (int64_t x = 0; x < dx; ++x) {
                    const float n = q[y * dx + x];
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
            float* sp = malloc(sizeof(float) * (size_t)dx);
            for (int64_t y = 0; y < dy; ++y) {
                if (p->speckle_sd > 0)
                    row_normals(seed ^ 0xA5A5A5A5DEADBEEFull, 0x632BE59BD9B4E019ull, chunked, z, y, dy, dx, sp);
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
                    if (p->speckle_sd > 0) s += (float)p->speckle_sd * sp[x];
                    s = fminf(255.f, fmaxf(0.f, s));
                    o[y * dx + x] = (uint8_t)floorf(s + 0.5f);
                }
            }
            free(sp);
        }
        free(a);
        free(tmps);
    }
    free(sheet);
    return rc;
}

/* out: [z_end - z_begin][dy][dx]; 0 on success */
int fxo_synth_spiral(uint8_t* out, int64_t dz, int64_t dy, int64_t dx, const fxo_spiral* p, uint64_t seed,
                     int64_t z_begin, int64_t z_end) {
    return synth_spiral_impl(out, dz, dy, dx, p, seed, z_begin, z_end, 0);
}

/* the same with the noise keyed per 64^3 chunk (the out-of-core workload's volume) */
int fxo_synth_spiral_chunked(uint8_t* out, int64_t dz, int64_t dy, int64_t dx, const fxo_spiral* p, uint64_t seed,
                             int64_t z_begin, int64_t z_end) {
    return synth_spiral_impl(out, dz, dy, dx, p, seed, z_begin, z_end, 1);
}

/* ---- papyrus layer stacks with ink (the layer-stack workload's input) ---------------------------
 * The recipe (the benchmark's description of that input: papyrus fibre as anisotropic
 * Gaussian-filtered noise, a sparse ink blob mask adding a fixed intensity): white N(0, 1) noise
 * per voxel (PCG stream per (stack, z, y) row), separable Gaussian passes along x, y, then z
 * (radius ceil(3 sigma), normalised weights, edge clamp), rescaled to standard deviation sd
 * around mean by the filter's noise gain sqrt(sum kz^2 sum ky^2 sum kx^2); ink = the
 * floor(fraction * dy * dx) largest values of a 2D-filtered noise plane (PCG stream per
 * (stack, y) row), + ink_delta on every layer of those columns; clip [0, 255], round half up. */
typedef struct fxo_papyrus {
    double sigma_z, sigma_y, sigma_x, mean, sd, ink_sigma, ink_fraction, ink_delta;
} fxo_papyrus;

static int gauss_taps(double sigma, float* k) {
    const int r = sigma > 0 ? (int)ceil(3.0 * sigma) : 0;
    if (r > 63) return -1;
    if (!r) {
        k[0] = 1.f;
        return 0;
    }
    double s = 0;
    for (int i = -r; i <= r; ++i) s += exp(-0.5 * i * i / (sigma * sigma));
    for (int i = -r; i <= r; ++i) k[i + r] = (float)(exp(-0.5 * i * i / (sigma * sigma)) / s);
    return r;
}

static double sum_sq(const float* k, int r) {
    double s = 0;
    for (int i = 0; i < 2 * r + 1; ++i) s += (double)k[i] * k[i];
    return s;
}

static void filter_line(const float* src, float* dst, int64_t n, int64_t step, const float* k, int r) {
    for (int64_t i = 0; i < n; ++i) {
        float s = 0.f;
        for (int j = -r; j <= r; ++j) s += k[j + r] * src[clampi(i + j, 0, n - 1) * step];
        dst[i * step] = s;
    }
}

static int cmp_desc(const void* a, const void* b) {
    const float x = *(const float*)a, y = *(const float*)b;
    return x < y ? 1 : (x > y ? -1 : 0);
}

int fxo_synth_papyrus(uint8_t* out, uint8_t* ink, int64_t dz, int64_t dy, int64_t dx, const fxo_papyrus* p,
                      uint64_t seed, int64_t stack) {
    if (!out || !p || dz < 1 || dy < 1 || dx < 1 || stack < 0) return 1;
    float kz[127], ky[127], kx[127], ki[127];
    const int rz = gauss_taps(p->sigma_z, kz), ry = gauss_taps(p->sigma_y, ky), rx = gauss_taps(p->sigma_x, kx);
    const int ri = gauss_taps(p->ink_sigma, ki);
    if (rz < 0 || ry < 0 || rx < 0 || ri < 0) return 1;
    const int64_t plane = dy * dx, n = dz * plane;
    float* a = malloc(sizeof(float) * (size_t)n);
    float* b = malloc(sizeof(float) * (size_t)n);
    float* f = malloc(sizeof(float) * (size_t)plane);
    float* g = malloc(sizeof(float) * (size_t)plane);
    uint8_t* mask = calloc((size_t)plane, 1);
    if (!a || !b || !f || !g || !mask) {
        free(a), free(b), free(f), free(g), free(mask);
        return 1;
    }
#pragma omp parallel for schedule(static)
    for (int64_t z = 0; z < dz; ++z) {
        float* P = a + z * plane;
        float* Q = b + z * plane;
        for (int64_t y = 0; y < dy; ++y) {
            pcg_t r = pcg_seed(seed ^ 0x5EED0F1B4E5ull, (uint64_t)((stack * dz + z) * dy + y) + 0x2545F4914F6CDD1Dull);
            for (int64_t x = 0; x < dx; ++x) P[y * dx + x] = pcg_normal(&r);
        }
        for (int64_t y = 0; y < dy; ++y) filter_line(P + y * dx, Q + y * dx, dx, 1, kx, rx);
        for (int64_t x = 0; x < dx; ++x) filter_line(Q + x, P + x, dy, dx, ky, ry);
    }
#pragma omp parallel for schedule(static)
    for (int64_t y = 0; y < dy; ++y)
        for (int64_t x = 0; x < dx; ++x) filter_line(a + y * dx + x, b + y * dx + x, dz, plane, kz, rz);
    for (int64_t y = 0; y < dy; ++y) {
        pcg_t r = pcg_seed(seed ^ 0x1A4B1075ull, (uint64_t)(stack * dy + y) + 0x9E3779B97F4A7C15ull);
        for (int64_t x = 0; x < dx; ++x) f[y * dx + x] = pcg_normal(&r);
    }
    for (int64_t y = 0; y < dy; ++y) filter_line(f + y * dx, g + y * dx, dx, 1, ki, ri);
    for (int64_t x = 0; x < dx; ++x) filter_line(g + x, f + x, dy, dx, ki, ri);
    const int64_t kink = (int64_t)floor(p->ink_fraction * (double)plane);
    if (kink > 0) {
        memcpy(g, f, sizeof(float) * (size_t)plane);
        qsort(g, (size_t)plane, sizeof(float), cmp_desc);
        const float thr = g[kink - 1];
        for (int64_t i = 0; i < plane; ++i) mask[i] = f[i] >= thr ? 1 : 0;
    }
    if (ink) memcpy(ink, mask, (size_t)plane);
    const float scale = (float)(p->sd / sqrt(sum_sq(kz, rz) * sum_sq(ky, ry) * sum_sq(kx, rx)));
    const float mean = (float)p->mean, delta = (float)p->ink_delta;
#pragma omp parallel for schedule(static)
    for (int64_t z = 0; z < dz; ++z)
        for (int64_t i = 0; i < plane; ++i) {
            float s = mean + scale * b[z * plane + i];
            if (mask[i]) s += delta;
            s = fminf(255.f, fmaxf(0.f, s));
            out[z * plane + i] = (uint8_t)floorf(s + 0.5f);
        }
    free(a), free(b), free(f), free(g), free(mask);
    return 0;
}
