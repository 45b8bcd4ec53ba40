// fenix_b200/ml/tiling.hpp — sliding-window tiling math: tile start positions, the Gaussian
// importance window, and the accumulated (factorised) blend-weight profile of one axis.
// Header-only, no CUDA. These three functions decide where every tile lands and how much each
// voxel weighs, so their results must equal the reference's bit for bit; each keeps the
// reference's expression order (the weight profile's sequential float sums included).
#pragma once

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

namespace fenix::ml {

using s64 = std::int64_t;

// exp(-1/2 ((i - c)/sigma)^2) with c = (n-1)/2, sigma = n/8, divided by its maximum, floored at
// 0.1 (src/ml/tiling.hpp:16-27). Evaluated in double, stored as float.
inline std::vector<float> gaussian1d(int n) {
    const double c = (n - 1) / 2.0, sigma = n / 8.0;
    std::vector<float> w(static_cast<std::size_t>(n > 0 ? n : 0));
    double mx = 0.0;
    for (int i = 0; i < n; ++i) {
        const double dd = (i - c) / sigma;
        w[static_cast<std::size_t>(i)] = static_cast<float>(std::exp(-0.5 * dd * dd));
        mx = std::max(mx, static_cast<double>(w[static_cast<std::size_t>(i)]));
    }
    for (auto& v : w) v = std::max(static_cast<float>(v / mx), 0.1f);
    return w;
}

// 0, step, 2 step, ... with the last start clamped to dim - patch; dim <= patch gives {0}
// (src/ml/tiling.hpp:32-42). step = max(1, (s64)(patch * (1 - overlap))).
inline std::vector<s64> tile_starts(s64 dim, int patch, double overlap) {
    std::vector<s64> starts;
    if (dim <= patch) {
        starts.push_back(0);
        return starts;
    }
    const s64 step = std::max<s64>(1, static_cast<s64>(patch * (1.0 - overlap)));
    for (s64 s = 0;; s += step) {
        const s64 clamped = std::min(s, dim - patch);
        if (starts.empty() || starts.back() != clamped) starts.push_back(clamped);
        if (clamped == dim - patch) break;
    }
    return starts;
}

// For each coordinate of the core span [c0, c0 + cn) of an axis of length dim: the sum of the
// window weights g[c - s0] of every start s0 covering it, accumulated in start order
// (src/ml/infer.hpp:499-509; with c0 = 0, cn = dim it is global_weight_profile,
// src/ml/global_accum.hpp:29-35).
inline std::vector<float> weight_profile(const std::vector<float>& g, const std::vector<s64>& starts, s64 c0, s64 cn,
                                         s64 dim, int patch) {
    std::vector<float> w(static_cast<std::size_t>(cn > 0 ? cn : 0), 0.0f);
    for (s64 s0 : starts)
        for (int i = 0; i < patch && s0 + i < dim; ++i) {
            const s64 gc = s0 + i;
            if (gc >= c0 && gc < c0 + cn) w[static_cast<std::size_t>(gc - c0)] += g[static_cast<std::size_t>(i)];
        }
    return w;
}

}  // namespace fenix::ml
