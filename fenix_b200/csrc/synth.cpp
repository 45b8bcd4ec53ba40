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

extern "C" int fx_synth_spiral(uint8_t* out, int64_t dz, int64_t dy, int64_t dx, const fx_spiral_params* prm,
                               uint64_t seed, int64_t z_begin, int64_t z_end) {
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
            for (int64_t y = 0; y < dy; ++y) {
                Pcg rng(seed, static_cast<uint64_t>(z * dy + y) + 0x9E3779B97F4A7C15ull);
                for (int64_t x = 0; x < dx; ++x) {
                    const float n = rng.normal();
                    p[y * dx + x] = sheet[y * dx + x]
                                        ? static_cast<float>(prm->sheet_mean + prm->sheet_sd * n)
                                        : static_cast<float>(prm->bg_mean + prm->bg_sd * n);
                }
            }
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
            for (int64_t y = 0; y < dy; ++y) {
                Pcg rng(seed ^ 0xA5A5A5A5DEADBEEFull, static_cast<uint64_t>(z * dy + y) + 0x632BE59BD9B4E019ull);
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
                    if (prm->speckle_sd > 0) s += static_cast<float>(prm->speckle_sd) * rng.normal();
                    s = std::min(255.f, std::max(0.f, s));
                    o[y * dx + x] = static_cast<uint8_t>(std::floor(s + 0.5f));
                }
            }
        });
    }
    return 0;
}
