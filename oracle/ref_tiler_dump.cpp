// ref_tiler_dump.cpp — prints the reference's own tiling results (tile_starts, gaussian1d and
// the accumulated weight profile, src/ml/tiling.hpp and src/ml/global_accum.hpp compiled from
// the reference sources) for a fixed list of cases, as hex floats, so the oracle and the
// product's host tiling can be compared bit for bit. Oracle tooling, not product code.
#include "ml/global_accum.hpp"
#include "ml/tiling.hpp"

#include <cstdio>

int main() {
    struct Case { long long dim; int patch; double ov; };
    const Case cases[] = {{64, 256, 0.5},  {256, 128, 0.5}, {300, 128, 0.5},  {1024, 128, 0.5}, {4096, 192, 0.5},
                          {2048, 192, 0.5}, {512, 256, 0.25}, {64, 64, 0.5},   {160, 64, 0.5},   {1000, 128, 0.25},
                          {130, 64, 0.5},  {384, 128, 0.5}, {200, 128, 0.75}, {129, 128, 0.5},  {192, 64, 0.0}};
    for (const Case& c : cases) {
        const auto s = fenix::ml::tile_starts(c.dim, c.patch, c.ov);
        std::printf("starts %lld %d %.17g :", c.dim, c.patch, c.ov);
        for (auto v : s) std::printf(" %lld", static_cast<long long>(v));
        std::printf("\n");
        const auto g = fenix::ml::gaussian1d(c.patch);
        const auto w = fenix::ml::global_weight_profile(g, s, c.dim, c.patch);
        std::printf("profile %lld %d %.17g :", c.dim, c.patch, c.ov);
        for (float v : w) std::printf(" %a", static_cast<double>(v));
        std::printf("\n");
    }
    const int ns[] = {1, 2, 7, 8, 32, 64, 100, 128, 192, 256, 384};
    for (int n : ns) {
        const auto g = fenix::ml::gaussian1d(n);
        std::printf("gauss %d :", n);
        for (float v : g) std::printf(" %a", static_cast<double>(v));
        std::printf("\n");
    }
    return 0;
}
