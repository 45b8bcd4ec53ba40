// synth.cpp — deterministic synthetic CT generator: an Archimedean spiral sheet (the scroll
// surface the net predicts) extruded along z, sheet/background intensities drawn from normal
// distributions, separable Gaussian blur, optional speckle noise after the blur, clip to
// [0, 255]. Test-input generation for the parity tests and the benchmark, not part of the
// inference path. Any z-range regenerates independently: every voxel's noise comes from a
// PCG32 stream keyed by its (z, y) row, so slabs match the whole volume byte for byte.
#include "fenix_b200_synth.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <functional>
#include <thread>
#include <vector>

namespace {

// PCG-XSH-RR 64/32 (M. O'Neill, "PCG: A Family of Simple Fast Space-Efficient Statistically
// Good Algorithms for Random Number Generation", 2014), with the usual seeding sequence.
struct Pcg {
    uint64_t state = 0, inc = 1;
    Pcg(uint64_t seed, uint64_t stream) {
        inc = (stream << 1u) | 1u;
        state = 0;
        next();
        state += seed;
        next();
    }
    uint32_t next() {
        const uint64_t old = state;
        state = old * 6364136223846793005ULL + inc;
        const uint32_t xs = static_cast<uint32_t>(((old >> 18u) ^ old) >> 27u);
        const uint32_t rot = static_cast<uint32_t>(old >> 59u);
        return (xs >> rot) | (xs << ((~rot + 1u) & 31u));
    }
    float uniform() { return static_cast<float>(next() >> 8) * (1.0f / 16777216.0f); }
    // Box-Muller, one normal per two uniforms.
    float normal() {
        const float u1 = std::max(uniform(), 1e-7f), u2 = uniform();
        return std::sqrt(-2.0f * std::log(u1)) * std::cos(6.28318530718f * u2);
    }
};

}  // namespace

namespace {
void parallel_rows(int64_t n, const std::function<void(int64_t)>& f) {
    unsigned nt = std::max(1u, std::thread::hardware_concurrency());
    nt = static_cast<unsigned>(std::min<int64_t>(nt, std::max<int64_t>(1, n)));
    std::vector<std::thread> th;
    for (unsigned t = 0; t < nt; ++t)
        th.emplace_back([&, t] {
            for (int64_t i = t; i < n; i += nt) f(i);
        });
    for (auto& x : th) x.join();
}

// Radial distance from (y, x) to the nearest turn of the spiral r = b * phi (phi >= 0),
// b = pitch / (2 pi), centred on the (y, x) plane's centre.
float sheet_distance(double y, double x, double cy, double cx, double pitch) {
    const double ry = y - cy, rx = x - cx;
    const double r = std::sqrt(ry * ry + rx * rx);
    const double th = std::atan2(ry, rx) + M_PI;  // [0, 2 pi]
    const double b = pitch / (2.0 * M_PI);
    // turns k >= 0 at radii b (th + 2 pi k)
    double k = std::round((r / b - th) / (2.0 * M_PI));
    if (k < 0) k = 0;
    return static_cast<float>(std::fabs(r - b * (th + 2.0 * M_PI * k)));
}
}  // namespace

namespace {
// The normals of one (z, y) row into f[0, dx): one PCG stream per row (row keying), or one per
// 64-voxel run of the row inside its 64^3 chunk, keyed by the chunk's index and the run's (z, y)
// within it (chunk keying: any chunk regenerates from its own streams).
template <class F>
void row_normals(uint64_t seed, uint64_t salt, bool chunked, int64_t z, int64_t y, int64_t dy, int64_t dx, F&& put) {
    if (!chunked) {
        Pcg rng(seed, static_cast<uint64_t>(z * dy + y) + salt);
        for (int64_t x = 0; x < dx; ++x) put(x, rng.normal());
        return;
    }
    const int64_t ncy = (dy + 63) / 64, ncx = (dx + 63) / 64;
    for (int64_t x0 = 0; x0 < dx; x0 += 64) {
        const uint64_t chunk = static_cast<uint64_t>(((z >> 6) * ncy + (y >> 6)) * ncx + (x0 >> 6));
        Pcg rng(seed, ((chunk << 12) | (static_cast<uint64_t>(z & 63) << 6) | static_cast<uint64_t>(y & 63)) + salt);
        for (int64_t x = x0; x < std::min(dx, x0 + 64); ++x) put(x, rng.normal());
    }
}

int synth_spiral_impl(uint8_t* out, int64_t dz, int64_t dy, int64_t dx, const fx_spiral_params* prm, uint64_t seed,
                      int64_t z_begin, int64_t z_end, bool chunked) {
    if (!out || !prm || dz < 1 || dy < 1 || dx < 1 || z_begin < 0 || z_end > dz || z_begin >= z_end) return 1;
    const double cy = (dy - 1) / 2.0, cx = (dx - 1) / 2.0;
    const int rad = prm->blur_sigma > 0 ? static_cast<int>(std::ceil(3.0 * prm->blur_sigma)) : 0;
    std::vector<float> k(2 * rad + 1, 1.f);
    if (rad) {
        double s = 0;
        for (int i = -rad; i <= rad; ++i) s += std::exp(-0.5 * i * i / (prm->blur_sigma * prm->blur_sigma));
        for (int i = -rad; i <= rad; ++i)
            k[i + rad] = static_cast<float>(std::exp(-0.5 * i * i / (prm->blur_sigma * prm->blur_sigma)) / s);
    }
    // sheet mask of one (y, x) plane (the sheet is extruded along z)
    std::vector<uint8_t> sheet(static_cast<size_t>(dy * dx));
    parallel_rows(dy, [&](int64_t y) {
        for (int64_t x = 0; x < dx; ++x)
            sheet[y * dx + x] = sheet_distance(static_cast<double>(y), static_cast<double>(x), cy, cx, prm->pitch) <
                                        0.5 * prm->thickness
                                    ? 1
                                    : 0;
    });
    const int64_t plane = dy * dx;
    const int64_t chunk = 32;
    for (int64_t c0 = z_begin; c0 < z_end; c0 += chunk) {
        const int64_t c1 = std::min(z_end, c0 + chunk);
        const int64_t g0 = std::max<int64_t>(0, c0 - rad), g1 = std::min<int64_t>(dz, c1 + rad);
        const int64_t ng = g1 - g0;
        std::vector<float> a(static_cast<size_t>(ng * plane));
        // raw intensities, then blur along x and y per plane
        parallel_rows(ng, [&](int64_t zi) {
            const int64_t z = g0 + zi;
            float* p = a.data() + zi * plane;
            for (int64_t y = 0; y < dy; ++y)
                row_normals(seed, 0x9E3779B97F4A7C15ull, chunked, z, y, dy, dx, [&](int64_t x, float n) {
                    p[y * dx + x] = sheet[y * dx + x]
                                        ? static_cast<float>(prm->sheet_mean + prm->sheet_sd * n)
                                        : static_cast<float>(prm->bg_mean + prm->bg_sd * n);
                });
            if (!rad) return;
            std::vector<float> tmp(static_cast<size_t>(plane));
            for (int64_t y = 0; y < dy; ++y)
                for (int64_t x = 0; x < dx; ++x) {
                    float s = 0.f;
                    for (int i = -rad; i <= rad; ++i) s += k[i + rad] * p[y * dx + std::clamp<int64_t>(x + i, 0, dx - 1)];
                    tmp[y * dx + x] = s;
                }
            for (int64_t y = 0; y < dy; ++y)
                for (int64_t x = 0; x < dx; ++x) {
                    float s = 0.f;
                    for (int i = -rad; i <= rad; ++i) s += k[i + rad] * tmp[std::clamp<int64_t>(y + i, 0, dy - 1) * dx + x];
                    p[y * dx + x] = s;
                }
        });
        // blur along z, speckle, clip, round
        parallel_rows(c1 - c0, [&](int64_t zo) {
            const int64_t z = c0 + zo;
            uint8_t* o = out + (z - z_begin) * plane;
            std::vector<float> sp(static_cast<size_t>(dx), 0.f);
            for (int64_t y = 0; y < dy; ++y) {
                if (prm->speckle_sd > 0)
                    row_normals(seed ^ 0xA5A5A5A5DEADBEEFull, 0x632BE59BD9B4E019ull, chunked, z, y, dy, dx,
                                [&](int64_t x, float n) { sp[x] = n; });
                for (int64_t x = 0; x < dx; ++x) {
                    float s;
                    if (rad) {
                        s = 0.f;
                        for (int i = -rad; i <= rad; ++i) {
                            const int64_t zz = std::clamp<int64_t>(z + i, 0, dz - 1);
                            s += k[i + rad] * a[(zz - g0) * plane + y * dx + x];
                        }
                    } else {
                        s = a[(z - g0) * plane + y * dx + x];
                    }
                    if (prm->speckle_sd > 0) s += static_cast<float>(prm->speckle_sd) * sp[x];
                    s = std::min(255.f, std::max(0.f, s));
                    o[y * dx + x] = static_cast<uint8_t>(std::floor(s + 0.5f));
                }
            }
        });
    }
    return 0;
}
}  // namespace

extern "C" int fx_synth_spiral(uint8_t* out, int64_t dz, int64_t dy, int64_t dx, const fx_spiral_params* prm,
                               uint64_t seed, int64_t z_begin, int64_t z_end) {
    return synth_spiral_impl(out, dz, dy, dx, prm, seed, z_begin, z_end, false);
}

extern "C" int fx_synth_spiral_chunked(uint8_t* out, int64_t dz, int64_t dy, int64_t dx, const fx_spiral_params* prm,
                                       uint64_t seed, int64_t z_begin, int64_t z_end) {
    return synth_spiral_impl(out, dz, dy, dx, prm, seed, z_begin, z_end, true);
}

namespace {
// Normalised Gaussian weights exp(-i^2 / 2 sigma^2), i in [-r, r], r = ceil(3 sigma) (r = 0: {1}).
std::vector<float> gauss_taps(double sigma) {
    const int r = sigma > 0 ? static_cast<int>(std::ceil(3.0 * sigma)) : 0;
    std::vector<float> k(2 * r + 1, 1.f);
    if (!r) return k;
    double s = 0;
    for (int i = -r; i <= r; ++i) s += std::exp(-0.5 * i * i / (sigma * sigma));
    for (int i = -r; i <= r; ++i) k[i + r] = static_cast<float>(std::exp(-0.5 * i * i / (sigma * sigma)) / s);
    return k;
}

double sum_sq(const std::vector<float>& k) {
    double s = 0;
    for (float v : k) s += static_cast<double>(v) * v;
    return s;
}

// One separable pass over rows of n elements spaced `step` apart: dst[i] = sum_j k[j] src[clamp(i + j - r)].
void filter_line(const float* src, float* dst, int64_t n, int64_t step, const std::vector<float>& k) {
    const int r = static_cast<int>(k.size() / 2);
    for (int64_t i = 0; i < n; ++i) {
        float s = 0.f;
        for (int j = -r; j <= r; ++j) s += k[j + r] * src[std::clamp<int64_t>(i + j, 0, n - 1) * step];
        dst[i * step] = s;
    }
}
}  // namespace

extern "C" int fx_synth_papyrus(uint8_t* out, uint8_t* ink, int64_t dz, int64_t dy, int64_t dx,
                                const fx_papyrus_params* prm, uint64_t seed, int64_t stack) {
    if (!out || !prm || dz < 1 || dy < 1 || dx < 1 || stack < 0 || prm->sigma_z < 0 || prm->sigma_y < 0 ||
        prm->sigma_x < 0 || prm->ink_sigma < 0 || !(prm->ink_fraction >= 0 && prm->ink_fraction <= 1))
        return 1;
    const auto kz = gauss_taps(prm->sigma_z), ky = gauss_taps(prm->sigma_y), kx = gauss_taps(prm->sigma_x);
    const auto ki = gauss_taps(prm->ink_sigma);
    const int64_t plane = dy * dx, n = dz * plane;
    std::vector<float> a(static_cast<size_t>(n)), b(static_cast<size_t>(n));
    // texture noise, then x and y passes per layer
    parallel_rows(dz, [&](int64_t z) {
        float* p = a.data() + z * plane;
        float* q = b.data() + z * plane;
        for (int64_t y = 0; y < dy; ++y) {
            Pcg rng(seed ^ 0x5EED0F1B4E5ull, static_cast<uint64_t>((stack * dz + z) * dy + y) + 0x2545F4914F6CDD1Dull);
            for (int64_t x = 0; x < dx; ++x) p[y * dx + x] = rng.normal();
        }
        for (int64_t y = 0; y < dy; ++y) filter_line(p + y * dx, q + y * dx, dx, 1, kx);
        for (int64_t x = 0; x < dx; ++x) filter_line(q + x, p + x, dy, dx, ky);
    });
    // z pass
    parallel_rows(dy, [&](int64_t y) {
        for (int64_t x = 0; x < dx; ++x) filter_line(a.data() + y * dx + x, b.data() + y * dx + x, dz, plane, kz);
    });
    // ink plane: noise, 2D filter, the top floor(fraction * dy * dx) columns
    std::vector<float> f(static_cast<size_t>(plane)), g(static_cast<size_t>(plane));
    for (int64_t y = 0; y < dy; ++y) {
        Pcg rng(seed ^ 0x1A4B1075ull, static_cast<uint64_t>(stack * dy + y) + 0x9E3779B97F4A7C15ull);
        for (int64_t x = 0; x < dx; ++x) f[y * dx + x] = rng.normal();
    }
    for (int64_t y = 0; y < dy; ++y) filter_line(f.data() + y * dx, g.data() + y * dx, dx, 1, ki);
    for (int64_t x = 0; x < dx; ++x) filter_line(g.data() + x, f.data() + x, dy, dx, ki);
    const int64_t kink = static_cast<int64_t>(std::floor(prm->ink_fraction * static_cast<double>(plane)));
    std::vector<uint8_t> mask(static_cast<size_t>(plane), 0);
    if (kink > 0) {
        std::vector<float> srt(f);
        std::nth_element(srt.begin(), srt.begin() + (kink - 1), srt.end(), std::greater<float>());
        const float thr = srt[static_cast<size_t>(kink - 1)];
        for (int64_t i = 0; i < plane; ++i) mask[i] = f[i] >= thr ? 1 : 0;
    }
    if (ink) std::copy(mask.begin(), mask.end(), ink);
    const float scale = static_cast<float>(prm->sd / std::sqrt(sum_sq(kz) * sum_sq(ky) * sum_sq(kx)));
    const float mean = static_cast<float>(prm->mean), delta = static_cast<float>(prm->ink_delta);
    parallel_rows(dz, [&](int64_t z) {
        for (int64_t i = 0; i < plane; ++i) {
            float s = mean + scale * b[z * plane + i];
            if (mask[i]) s += delta;
            s = std::min(255.f, std::max(0.f, s));
            out[z * plane + i] = static_cast<uint8_t>(std::floor(s + 0.5f));
        }
    });
    return 0;
}
