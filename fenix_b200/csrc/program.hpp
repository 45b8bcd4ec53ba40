// program.hpp — host-side compiler from one convolution (taps x row offsets over the padded
// group-plane layout) to the stage/MMA program and packed weights that conv_tc_kernel runs.
#pragma once

#include "conv_tc.cuh"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <map>
#include <string>
#include <vector>

namespace fxh {

struct Tap {
    int src;      // source array index (ConvParams::src)
    int64_t off;  // row offset relative to the output row
    int wkey;     // weight tap id passed to the weight accessor
    int window;   // taps with the same window share one staged run of rows
};

struct ProgramSpec {
    int optype = 0;    // fxk::OpType of the packed weights: 0 bf16, 1 e4m3, 2 f16
    int G = 0;         // input groups (16 bytes each)
    int cg = 8;        // channels per group: 8 (bf16) or 16 (e4m3)
    int elem = 2;      // bytes per element
    int N_total = 0;   // output columns
    int N_tile = 0;    // columns per work unit
    int R = 1;         // M blocks per unit
    int block_rows = 128;  // window rows advanced per M block (126 with the x-tap fold)
    std::vector<Tap> taps;
    // z-plane fold (3x3x3 stride 1): the R M blocks of a unit lie one z plane apart, each stage
    // holds one input plane's window, and its A tiles feed up to three blocks (taps kz = 0, 1, 2);
    // the weights stay resident in shared memory. zWp / zP2: padded row and plane of the grid.
    bool zfold = false;
    int64_t zWp = 0, zP2 = 0;
    int zsegs = 2;  // z-plane fold: adjacent 128-row segments per unit (R = planes per segment)
    // B value for output column n, input channel ci (0 <= ci < G*cg), tap key
    std::function<float(int n, int ci, int wkey)> wval;
    int smem_total = 212 * 1024;  // stage buffers; the control block takes the rest
};

struct Program {
    std::vector<fxk::ConvStage> stages;
    std::vector<fxk::ConvMma> mmas;
    std::vector<uint8_t> wpack;  // n_tiles blocks of wtile_bytes
    int64_t wtile_bytes = 0;
    int stage_bytes = 0, stage_a_bytes = 0, n_pipe = 0;
    int n_tiles = 0;
    int bres_bytes = 0;  // z-plane fold: resident weights (all taps), 0 otherwise
    int zkstride = 0;    // z-plane fold: bytes between the weight blocks of taps kz and kz + 1
};

// e4m3 encode with round-to-nearest-even and saturation to +-448 (finite), host side.
inline uint8_t float_to_e4m3(float f) {
    if (std::isnan(f)) return 0x7f;
    uint8_t sign = std::signbit(f) ? 0x80 : 0x00;
    float a = std::fabs(f);
    if (a >= 448.f) return sign | 0x7e;  // max finite 448
    if (a < std::ldexp(1.f, -10)) {  // below half of the smallest subnormal (2^-9)
        return sign;
    }
    // candidates: enumerate all 126 finite positive codes and pick nearest (ties to even code)
    static float table[127];
    static bool init = false;
    if (!init) {
        for (int c = 0; c < 127; ++c) {
            const int e = (c >> 3) & 0xf, m = c & 7;
            table[c] = e == 0 ? std::ldexp(static_cast<float>(m), -9) : std::ldexp(1.f + m / 8.f, e - 7);
        }
        init = true;
    }
    int lo = 0, hi = 126;
    while (hi - lo > 1) {
        const int mid = (lo + hi) / 2;
        if (table[mid] <= a) lo = mid; else hi = mid;
    }
    int best;
    const float dl = a - table[lo], dh = table[hi] - a;
    if (dl < dh) best = lo;
    else if (dh < dl) best = hi;
    else best = (lo & 1) ? hi : lo;
    return sign | static_cast<uint8_t>(best);
}

// IEEE binary16, round to nearest even, saturated to +-65504.
inline uint16_t float_to_f16(float f) {
    if (std::isnan(f)) return 0x7e00;
    f = std::fmax(-65504.f, std::fmin(65504.f, f));
    uint32_t u;
    std::memcpy(&u, &f, 4);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const float a = std::fabs(f);
    if (a < std::ldexp(1.f, -25)) return static_cast<uint16_t>(sign);  // rounds to zero
    if (a < std::ldexp(1.f, -14)) {  // subnormal: multiples of 2^-24
        const float q = a * 16777216.f;  // exact
        float r = std::nearbyint(q);     // default rounding mode: nearest even
        return static_cast<uint16_t>(sign | static_cast<uint32_t>(r));
    }
    int e;
    const float m = std::frexp(a, &e);  // a = m * 2^e, m in [0.5, 1)
    // 11 significant bits
    float sig = std::nearbyint(std::ldexp(m, 11));  // in [1024, 2048]
    if (sig >= 2048.f) {
        sig = 1024.f;
        ++e;
    }
    const uint32_t exp = static_cast<uint32_t>(e - 1 + 15);
    if (exp >= 31) return static_cast<uint16_t>(sign | 0x7bffu);
    return static_cast<uint16_t>(sign | (exp << 10) | (static_cast<uint32_t>(sig) & 0x3ffu));
}

inline uint16_t float_to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return static_cast<uint16_t>(u >> 16);
}

// v rounded to the 16-bit operand type q (2 f16, else bf16), as the packer rounds it.
inline float round16_host(float v, int q) {
    uint32_t u;
    if (q == 2) {
        const uint16_t h = float_to_f16(v);
        const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
        const float a = e == 0 ? std::ldexp(static_cast<float>(m), -24) : std::ldexp(1.f + m / 1024.f, static_cast<int>(e) - 15);
        return (h & 0x8000u) ? -a : a;
    }
    u = static_cast<uint32_t>(float_to_bf16(v)) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// A / B smem offsets of one MMA packed into descriptor low words (see fxk::ConvMma).
inline fxk::ConvMma pack_mma(int64_t a_off, int64_t lbo, int64_t b_off) {
    fxk::ConvMma m{};
    m.a = (static_cast<uint32_t>(lbo >> 4) << 16) | static_cast<uint32_t>(a_off >> 4);
    m.b = static_cast<uint32_t>(b_off >> 4);
    return m;
}

// z-plane fold program (see ProgramSpec::zfold). Stage j = 0 .. R+1 stages input plane
// z0 + j - 1 of the unit: rows [-(Wp+1), 128 S + Wp + 1) around the unit's S adjacent (y, x)
// segments, all groups. Its MMA entries are the 9 (ky, kx) shifts x group pairs; the kernel issues
// each entry for every segment (A + 128 rows per segment), with the taps kz of 0 <= j - kz < R
// stacked along N into blocks (segment, j - kz); the weights of (entry, kz) start at
// entry.b + kz * zkstride of the resident region, zkstride = N_tile rows of 16 B.
// Returns "" on success.
inline std::string build_zfold_program(const ProgramSpec& s, Program& pg) {
    if (s.N_tile != s.N_total || s.N_tile > 256 || s.N_tile % 16) return "zfold: one N tile of at most 256 columns";
    if (s.G % 2) return "zfold: group count must be even";
    const int64_t Wp = s.zWp;
    const int rows = static_cast<int>(128 * s.zsegs + 2 * (Wp + 1));
    const int bblk = s.N_tile * 32;
    const int nent = 9 * (s.G / 2);
    pg.bres_bytes = 3 * nent * bblk;
    pg.zkstride = s.N_tile * 16;  // tap kz -> kz + 1 within an entry's block
    const int sb = rows * s.G * 16;
    pg.stage_bytes = (sb + 127) / 128 * 128;
    pg.stage_a_bytes = pg.stage_bytes;
    const int avail = s.smem_total - pg.bres_bytes;
    pg.n_pipe = std::min(8, avail / std::max(pg.stage_bytes, 1));
    if (pg.n_pipe < 3) return "zfold: resident weights leave fewer than 3 stages";
    pg.n_tiles = 1;
    pg.stages.clear();
    pg.mmas.clear();
    for (int ky = 0; ky < 3; ++ky)
        for (int kx = 0; kx < 3; ++kx)
            for (int gp = 0; gp < s.G; gp += 2) {
                const int e = static_cast<int>(pg.mmas.size());
                const int64_t a_off = static_cast<int64_t>(gp) * rows * 16 + (ky * Wp + kx) * 16;
                pg.mmas.push_back(pack_mma(a_off, static_cast<int64_t>(rows) * 16, static_cast<int64_t>(e) * 3 * bblk));
            }
    for (int j = 0; j < s.R + 2; ++j) {
        fxk::ConvStage st{};
        st.src = 0;
        st.row_off = static_cast<int32_t>((j - 1) * s.zP2 - (Wp + 1));
        st.rows = rows;
        st.g0 = 0;
        st.ng = s.G;
        st.b_off = 0;
        st.b_bytes = 0;
        st.mma_begin = 0;
        st.mma_count = nent;
        pg.stages.push_back(st);
    }
    for (const auto& m : pg.mmas)
        if ((m.a & 0xFFFFu) >= 0x4000u || (m.a >> 16) >= 0x4000u || m.b >= 0x4000u) return "zfold: smem offset overflow";
    // resident weights: one block per (ky, kx, group pair) entry, [K half][kz][N_tile][16 B]: the
    // three kz taps are consecutive B rows, so one MMA of N = k N_tile covers k adjacent taps
    pg.wtile_bytes = pg.bres_bytes;
    pg.wpack.assign(static_cast<size_t>(pg.bres_bytes), 0);
    for (int kz = 0; kz < 3; ++kz)
        for (int e = 0; e < nent; ++e) {
            const int kyx = e / (s.G / 2), gp = (e % (s.G / 2)) * 2;
            const int wk = kz * 9 + kyx;  // ky * 3 + kx == kyx
            uint8_t* blk = pg.wpack.data() + static_cast<size_t>(e) * 3 * bblk;
            for (int h = 0; h < 2; ++h)
                for (int n = 0; n < s.N_tile; ++n) {
                    uint8_t* row = blk + ((static_cast<size_t>(h) * 3 + kz) * s.N_tile + n) * 16;
                    for (int jj = 0; jj < s.cg; ++jj) {
                        const float v = s.wval(n, (gp + h) * s.cg + jj, wk);
                        if (s.elem == 2) {
                            const uint16_t b = s.optype == 2 ? float_to_f16(v) : float_to_bf16(v);
                            std::memcpy(row + 2 * jj, &b, 2);
                        } else {
                            row[jj] = float_to_e4m3(v);
                        }
                    }
                }
        }
    return {};
}

// Returns "" on success.
inline std::string build_program(const ProgramSpec& s, Program& pg) {
    if (s.zfold) return build_zfold_program(s, pg);
    if (s.N_tile <= 0 || s.N_tile % 16 || s.N_total % s.N_tile) return "program: bad N tiling";
    if (s.N_tile > 256 && s.N_tile != 320) return "program: N tile > 256 must be 320";
    if (s.G % 2) return "program: group count must be even";
    const int Mtot = s.block_rows * (s.R - 1) + 128;  // rows spanned by a unit's M blocks
    // windows
    std::map<int, std::vector<Tap>> win;
    for (const Tap& t : s.taps) win[t.window].push_back(t);
    struct W {
        int src;
        int64_t lo, hi;
        std::vector<Tap> taps;
    };
    std::vector<W> ws;
    int max_rows = 0, max_taps = 0;
    for (auto& kv : win) {
        W w;
        w.src = kv.second[0].src;
        w.taps = kv.second;
        std::sort(w.taps.begin(), w.taps.end(), [](const Tap& a, const Tap& b) { return a.off < b.off; });
        w.lo = w.taps.front().off;
        w.hi = w.taps.back().off;
        for (auto& t : w.taps)
            if (t.src != w.src) return "program: window mixes sources";
        max_rows = std::max<int>(max_rows, static_cast<int>(Mtot + (w.hi - w.lo)));
        max_taps = std::max<int>(max_taps, static_cast<int>(w.taps.size()));
        ws.push_back(std::move(w));
    }
    // groups per stage: largest that keeps >= 3 stages in the smem budget (>= 2 as a fallback)
    const int bblk = s.N_tile * 32;  // bytes of one MMA's B block
    auto stage_bytes_for = [&](int gc) {
        const int nm = max_taps * (gc / 2);
        return max_rows * gc * 16 + nm * bblk;
    };
    int gc = 2;
    for (int c = s.G; c >= 2; c -= 2)
        if (stage_bytes_for(c) * 3 <= s.smem_total) {
            gc = c;
            break;
        }
    int sb = stage_bytes_for(gc);
    int n_pipe = std::min(8, s.smem_total / sb);
    if (n_pipe < 2) return "program: stage does not fit in shared memory (" + std::to_string(sb) + " bytes)";
    pg.stage_bytes = (sb + 127) / 128 * 128;
    pg.stage_a_bytes = max_rows * gc * 16;
    n_pipe = std::min(8, s.smem_total / pg.stage_bytes);
    pg.n_pipe = n_pipe;
    pg.n_tiles = s.N_total / s.N_tile;
    pg.stages.clear();
    pg.mmas.clear();

    // B blocks are recorded as (tap A, tap B or -1, group pair) and packed per N tile below.
    struct BRec {
        int wk0, wk1;  // tap keys for the two K-halves (-1 = zeros)
        int g0, g1;    // input groups of the two K-halves
    };
    std::vector<BRec> brecs;
    int32_t boff = 0;
    for (const W& w : ws) {
        const int rows = static_cast<int>(Mtot + (w.hi - w.lo));
        for (int g0 = 0; g0 < s.G; g0 += gc) {
            const int ng = std::min(gc, s.G - g0);
            fxk::ConvStage st{};
            st.src = w.src;
            st.row_off = static_cast<int32_t>(w.lo);
            st.rows = rows;
            st.g0 = g0;
            st.ng = ng;
            st.b_off = boff;
            st.mma_begin = static_cast<int32_t>(pg.mmas.size());
            int32_t local_b = 0;
            for (const Tap& t : w.taps)
                for (int gp = g0; gp < g0 + ng; gp += 2) {
                    const int64_t a_off = static_cast<int64_t>(gp - g0) * rows * 16 + (t.off - w.lo) * 16;
                    pg.mmas.push_back(pack_mma(a_off, static_cast<int64_t>(rows) * 16, local_b));
                    brecs.push_back({t.wkey, t.wkey, gp, gp + 1});
                    local_b += bblk;
                }
            st.mma_count = static_cast<int32_t>(pg.mmas.size()) - st.mma_begin;
            st.b_bytes = local_b;
            boff += local_b;
            pg.stages.push_back(st);
        }
    }
    if (pg.stages.size() > static_cast<size_t>(fxk::kMaxStages) || pg.mmas.size() > static_cast<size_t>(fxk::kMaxMmas))
        return "program: " + std::to_string(pg.stages.size()) + " stages / " + std::to_string(pg.mmas.size()) +
               " MMAs exceed the kernel's program capacity";
    // every packed offset must fit its 14-bit descriptor field (smem < 256 KB)
    for (const auto& m : pg.mmas)
        if ((m.a & 0xFFFFu) >= 0x4000u || (m.a >> 16) >= 0x4000u || m.b >= 0x4000u) return "program: smem offset overflow";
    pg.wtile_bytes = boff;
    pg.wpack.assign(static_cast<size_t>(boff) * pg.n_tiles, 0);
    const int cg = s.cg;
    for (int nt = 0; nt < pg.n_tiles; ++nt) {
        uint8_t* tile = pg.wpack.data() + static_cast<size_t>(nt) * boff;
        for (size_t k = 0; k < brecs.size(); ++k) {
            const BRec& br = brecs[k];
            uint8_t* blk = tile + k * bblk;
            for (int h = 0; h < 2; ++h) {
                const int wk = h == 0 ? br.wk0 : br.wk1;
                const int g = h == 0 ? br.g0 : br.g1;
                if (wk < 0) continue;
                for (int n = 0; n < s.N_tile; ++n) {
                    const int col = nt * s.N_tile + n;
                    uint8_t* row = blk + (static_cast<size_t>(h) * s.N_tile + n) * 16;
                    for (int j = 0; j < cg; ++j) {
                        const float v = s.wval(col, g * cg + j, wk);
                        if (s.elem == 2) {
                            const uint16_t b = s.optype == 2 ? float_to_f16(v) : float_to_bf16(v);
                            std::memcpy(row + 2 * j, &b, 2);
                        } else {
                            row[j] = float_to_e4m3(v);
                        }
                    }
                }
            }
        }
    }
    return {};
}

}  // namespace fxh
