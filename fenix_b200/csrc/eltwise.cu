// eltwise.cu — HBM-bound kernels of the inference path (see eltwise.cuh).
#include "eltwise.cuh"
#include "counters.hpp"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <algorithm>

namespace fxk {

namespace {

constexpr int kEwThreads = 256;

__device__ __forceinline__ int64_t clamp64(int64_t v, int64_t lo, int64_t hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

// Edge-clamped voxel read, as the reference's dense filler does (core/volume.hpp at_clamped).
__device__ __forceinline__ uint8_t vol_at(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, int64_t z,
                                          int64_t y, int64_t x) {
    z = clamp64(z, 0, dz - 1);
    y = clamp64(y, 0, dy - 1);
    x = clamp64(x, 0, dx - 1);
    return __ldg(vol + (z * dy + y) * dx + x);
}

// Exact integer sum and sum of squares of a tile's u8 voxels (edge tiles clamp to the volume).
// A warp walks whole (z, y) lines of the tile, lanes across x: one 32-bit division per line.
template <bool HIST>
__global__ void tile_sums_kernel(const uint8_t* __restrict__ vol, int64_t dz, int64_t dy, int64_t dx,
                                 const TileOrigin* __restrict__ tiles, TileDims P, unsigned long long* sums,
                                 unsigned* __restrict__ hist) {
    const int b = blockIdx.y;
    __shared__ unsigned h[HIST ? 256 : 1];
    if (HIST) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) h[i] = 0u;
        __syncthreads();
    }
    const TileOrigin t = tiles[b];
    const bool inside = t.z0 + P.z <= dz && t.y0 + P.y <= dy && t.x0 + P.x <= dx;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    constexpr int kWarps = kEwThreads / 32;
    unsigned long long s1 = 0, s2 = 0;
    const uint32_t lines = static_cast<uint32_t>(P.z) * P.y;
    for (uint32_t line = blockIdx.x * kWarps + w; line < lines; line += gridDim.x * kWarps) {
        const int z = static_cast<int>(line / static_cast<uint32_t>(P.y));
        const int y = static_cast<int>(line - static_cast<uint32_t>(z) * P.y);
        const uint8_t* src = vol + ((t.z0 + z) * dy + (t.y0 + y)) * dx + t.x0;
        uint32_t a1 = 0, a2 = 0;  // one line: at most P.x * 255^2 < 2^32 for P.x <= 66051
        for (int x = lane; x < P.x; x += 32) {
            const uint32_t v = inside ? __ldg(src + x) : vol_at(vol, dz, dy, dx, t.z0 + z, t.y0 + y, t.x0 + x);
            a1 += v;
            a2 += v * v;
            if (HIST) atomicAdd(&h[v], 1u);
        }
        s1 += a1;
        s2 += a2;
    }
    for (int o = 16; o >= 1; o >>= 1) {
        s1 += __shfl_down_sync(0xffffffffu, s1, o);
        s2 += __shfl_down_sync(0xffffffffu, s2, o);
    }
    __shared__ unsigned long long r1[kWarps], r2[kWarps];
    if (lane == 0) {
        r1[w] = s1;
        r2[w] = s2;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long a = 0, c = 0;
        for (int i = 0; i < kWarps; ++i) {
            a += r1[i];
            c += r2[i];
        }
        atomicAdd(&sums[2 * b], a);
        atomicAdd(&sums[2 * b + 1], c);
    }
    if (HIST) {
        __syncthreads();
        for (int i = threadIdx.x; i < 256; i += blockDim.x)
            if (h[i]) atomicAdd(hist + static_cast<int64_t>(b) * 256 + i, h[i]);
    }
}

// Per-tile z-score table: lut[v] = (float)((v - mean) / sd) with mean = S/n and
// sd = sqrt(max(Q/n - mean*mean, 1e-12)), every step an explicitly rounded double op so no
// contraction changes the result (src/ml/infer.hpp:350-385).
__device__ __forceinline__ void build_lut(float* lut, unsigned long long S, unsigned long long Q, int64_t n) {
    const double dn = static_cast<double>(n);
    const double mean = __ddiv_rn(static_cast<double>(S), dn);
    const double var = __dsub_rn(__ddiv_rn(static_cast<double>(Q), dn), __dmul_rn(mean, mean));
    const double sd = __dsqrt_rn(var > 1e-12 ? var : 1e-12);
    for (int v = threadIdx.x; v < 256; v += blockDim.x)
        lut[v] = static_cast<float>(__ddiv_rn(__dsub_rn(static_cast<double>(v), mean), sd));
}

// Per-tile normalisation table of the u8 levels, one block of 256 threads per tile
// (src/ml/infer.hpp:350-385, norm_patch):
//  zscore   lut[v] = (float)((v - mean) / sd) from the exact sums (build_lut);
//  unit255  lut[v] = (float)v * (1 / 255) in f32;
//  pct_minmax  the reference's percentile bounds (infer.hpp:107-134): a 1024-bin histogram over
//    [min, max] of the tile, whose bin of each u8 level is (x - min) * ((1024 - 1) / (max - min)) in
//    f32, cut at the 0.5 / 99.5 percent counts, then lut[v] = clamp((v - lo) / (hi - lo), 0, 1) with
//    the reciprocal taken first as the reference does. The u8 histogram gives every bin count
//    exactly, so the table equals the per-voxel computation.
// const_flag[b] (when non-null) = 1 for a tile whose voxels all hold one value.
__global__ void tile_lut_kernel(const unsigned long long* __restrict__ sums, const unsigned* __restrict__ hist,
                                int64_t n, int norm, float* __restrict__ luts, uint8_t* __restrict__ const_flag) {
    const int b = blockIdx.x;
    float* lut = luts + static_cast<int64_t>(b) * 256;
    const unsigned long long S = sums[2 * b], Q = sums[2 * b + 1];
    if (const_flag && threadIdx.x == 0) {
        // constant <=> n Q == S^2 (128-bit products)
        const unsigned long long un = static_cast<unsigned long long>(n);
        const bool c = __umul64hi(un, Q) == __umul64hi(S, S) && un * Q == S * S;
        const_flag[b] = c ? 1 : 0;
    }
    if (norm == 0) {
        build_lut(lut, S, Q, n);
        return;
    }
    if (norm == 2) {
        lut[threadIdx.x] = __fmul_rn(static_cast<float>(threadIdx.x), 1.0f / 255.0f);
        return;
    }
    __shared__ float s_lo, s_inv;
    if (threadIdx.x == 0) {
        const unsigned* hc = hist + static_cast<int64_t>(b) * 256;
        int vmin = 255, vmax = 0;
        for (int v = 0; v < 256; ++v)
            if (hc[v]) {
                vmin = min(vmin, v);
                vmax = max(vmax, v);
            }
        const float mn = static_cast<float>(vmin), mx = static_cast<float>(vmax);
        float lo, hi;
        if (mx <= mn) {
            lo = mn;
            hi = __fadd_rn(mn, 1.0f);
        } else {
            const float inv = __fdiv_rn(1023.0f, __fsub_rn(mx, mn));
            const long long tlo = static_cast<long long>(0.5 / 100.0 * static_cast<double>(n));
            const long long thi = static_cast<long long>(99.5 / 100.0 * static_cast<double>(n));
            // cumulative count over the 1024 bins: the u8 levels land in non-decreasing bins
            long long c = 0;
            int blo = 0, bhi = 1023, v = vmin;
            for (int bin = 0; bin < 1024; ++bin) {
                while (v <= vmax && static_cast<int>(__fmul_rn(__fsub_rn(static_cast<float>(v), mn), inv)) == bin) {
                    c += hc[v];
                    ++v;
                }
                if (c <= tlo) blo = bin;
                if (c < thi) bhi = bin;
            }
            lo = __fadd_rn(mn, __fdiv_rn(static_cast<float>(blo), inv));
            hi = __fadd_rn(mn, __fdiv_rn(static_cast<float>(bhi + 1), inv));
            if (hi <= lo) hi = __fadd_rn(lo, 1.0f);
        }
        s_lo = lo;
        s_inv = __fdiv_rn(1.0f, __fsub_rn(hi, lo));
    }
    __syncthreads();
    const float r = __fmul_rn(__fsub_rn(static_cast<float>(threadIdx.x), s_lo), s_inv);
    lut[threadIdx.x] = fminf(fmaxf(r, 0.0f), 1.0f);
}

__global__ void tile_norm_kernel(const uint8_t* __restrict__ vol, int64_t dz, int64_t dy, int64_t dx,
                                 const TileOrigin* __restrict__ tiles, TileDims P,
                                 const unsigned long long* __restrict__ sums, const float* __restrict__ luts,
                                 uint8_t* __restrict__ l0,
                                 int64_t l0_batch_stride, int64_t l0_group_stride, int l0_type,
                                 float* __restrict__ f32_out, const uint8_t* __restrict__ tta) {
    const int b = blockIdx.y;
    __shared__ float lut[256];
    const int64_t n = P.count();
    if (luts) {
        for (int v = threadIdx.x; v < 256; v += blockDim.x) lut[v] = luts[static_cast<int64_t>(b) * 256 + v];
    } else {
        build_lut(lut, sums[2 * b], sums[2 * b + 1], n);
    }
    __syncthreads();
    const TileOrigin t = tiles[b];
    const int Hp = P.y + 2, Wp = P.x + 2;
    const bool inside = t.z0 + P.z <= dz && t.y0 + P.y <= dy && t.x0 + P.x <= dx;
    // a warp walks whole (z, y) lines, lanes across x: one 32-bit division per line
    const int lane = threadIdx.x & 31;
    constexpr int kWarps = kEwThreads / 32;
    const uint32_t lines = static_cast<uint32_t>(P.z) * P.y;
    for (uint32_t line = blockIdx.x * kWarps + (threadIdx.x >> 5); line < lines; line += gridDim.x * kWarps)
    for (int x = lane; x < P.x; x += 32) {
        const int z = static_cast<int>(line / static_cast<uint32_t>(P.y));
        const int y = static_cast<int>(line - static_cast<uint32_t>(z) * P.y);
        const int64_t i = static_cast<int64_t>(line) * P.x + x;
        float v[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int xx = x - 1 + k;
            if (xx < 0 || xx >= P.x) {
                v[k] = 0.f;
            } else {
                int sz = z, sy = y, sx = xx;  // source voxel of this member's frame voxel (cubic tiles)
                if (tta) tta_source(tta[b], P.x, z, y, xx, sz, sy, sx);
                const uint8_t u = inside ? __ldg(vol + ((t.z0 + sz) * dy + (t.y0 + sy)) * dx + (t.x0 + sx))
                                         : vol_at(vol, dz, dy, dx, t.z0 + sz, t.y0 + sy, t.x0 + sx);
                v[k] = lut[u];
            }
        }
        const int64_t row = (static_cast<int64_t>(z + 1) * Hp + (y + 1)) * Wp + (x + 1);
        if (l0) {
            uint4 c0, c1;
            first_layer_cells(v, l0_type, c0, c1);
            uint8_t* o = l0 + b * l0_batch_stride + row * 16;
            *reinterpret_cast<uint4*>(o) = c0;
            *reinterpret_cast<uint4*>(o + l0_group_stride) = c1;
        }
        if (f32_out) f32_out[b * n + i] = v[1];
    }
}

// Division by a divisor fixed at launch, by multiply and shift (Granlund & Montgomery, "Division
// by invariant integers using multiplication", 1994): n / d = (umulhi(n, m) + n) >> s, exact for
// n < 2^31 with s = ceil(log2 d) and m = floor(2^32 (2^s - d) / d) + 1.
struct FastDiv {
    uint32_t d, m, s;
};
FastDiv make_fastdiv(uint32_t d) {
    uint32_t s = 0;
    while ((1ull << s) < d) ++s;
    const uint64_t m = ((1ull << 32) * ((1ull << s) - d)) / d + 1;
    return {d, static_cast<uint32_t>(m), s};
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) { return (__umulhi(n, f.m) + n) >> f.s; }

// InstanceNorm statistics, two levels. Block (channel block, batch, slice) sums its slice of the
// records [B][nrec][C][2] in double and stores {Σ, Σ²} for 32 channels in work[B][S][C][2]; the
// last block of a (batch, channel block) to finish — counted in done[], which it resets — adds
// the S slices in slice order (the result does not depend on block scheduling) and writes
// ss[B][C][2] = {gamma * rstd, beta - mean * gamma * rstd}. With ratio, the records hold the
// channel's values divided by ratio[c]: the statistics of the true values are mean * r and
// var * r^2, and ss is written for the stored values (scale multiplied by r). Every record read
// is left at zero: the conv epilogue adds its next partial sums into it.
__global__ void __launch_bounds__(256) in_stats_kernel(float* __restrict__ partials, int nrec, int C, int S,
                                                       double count, const float* __restrict__ gamma,
                                                       const float* __restrict__ beta,
                                                       const float* __restrict__ ratio, float eps,
                                                       double* __restrict__ work, unsigned* __restrict__ done,
                                                       float* __restrict__ ss) {
    const int b = blockIdx.y, sl = blockIdx.z;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    const int r0 = static_cast<int>(static_cast<int64_t>(nrec) * sl / S);
    const int r1 = static_cast<int>(static_cast<int64_t>(nrec) * (sl + 1) / S);
    double a1 = 0.0, a2 = 0.0;
    if (c < C) {
        float2* base = reinterpret_cast<float2*>(partials) + static_cast<int64_t>(b) * nrec * C + c;
#pragma unroll 4
        for (int r = r0 + w; r < r1; r += 8) {
            const float2 v = __ldcg(base + static_cast<int64_t>(r) * C);
            a1 += v.x;
            a2 += v.y;
        }
        // then clear them (the next conv adds into them); apart from the loads so those stay batched
        for (int r = r0 + w; r < r1; r += 8) base[static_cast<int64_t>(r) * C] = make_float2(0.f, 0.f);
    }
    __shared__ double s1[8][32], s2[8][32];
    s1[w][lane] = a1;
    s2[w][lane] = a2;
    __syncthreads();
    if (w != 0) return;
    double t1 = 0.0, t2 = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        t1 += s1[i][lane];
        t2 += s2[i][lane];
    }
    double* wb = work + static_cast<int64_t>(b) * S * C * 2;
    if (c < C) {
        wb[(static_cast<int64_t>(sl) * C + c) * 2] = t1;
        wb[(static_cast<int64_t>(sl) * C + c) * 2 + 1] = t2;
    }
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    unsigned* cnt = done + b * gridDim.x + blockIdx.x;
    if (lane == 0) prev = atomicAdd(cnt, 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != static_cast<unsigned>(S - 1)) return;
    __threadfence();
    if (c < C) {
        double u1 = 0.0, u2 = 0.0;
        for (int k = 0; k < S; ++k) {
            u1 += __ldcg(wb + (static_cast<int64_t>(k) * C + c) * 2);
            u2 += __ldcg(wb + (static_cast<int64_t>(k) * C + c) * 2 + 1);
        }
        const double r = ratio ? static_cast<double>(ratio[c]) : 1.0;
        const double ms = u1 / count;
        double var = (u2 / count - ms * ms) * r * r;
        if (var < 0.0) var = 0.0;
        const double mean = ms * r;
        const double rstd = 1.0 / sqrt(var + static_cast<double>(eps));
        const double sc = static_cast<double>(gamma ? gamma[c] : 1.f) * rstd;
        const double sh = static_cast<double>(beta ? beta[c] : 0.f) - mean * sc;
        ss[(static_cast<int64_t>(b) * C + c) * 2 + 0] = static_cast<float>(sc * r);
        ss[(static_cast<int64_t>(b) * C + c) * 2 + 1] = static_cast<float>(sh);
    }
    if (lane == 0) *cnt = 0u;
}

__device__ __forceinline__ void store_dest(const NormDest& d, int b, int gout, int64_t row, int zp, int yp, int xp,
                                           const float* y, int n) {
    if (!d.ptr) return;
    int64_t off;
    if (d.phase) {
        off = phase_cell_offset(d.phase, zp, yp, xp, d.pHp, d.pWp, d.phase_stride);
    } else {
        off = row * 16;
    }
    uint8_t* o = d.ptr + b * d.batch_stride + gout * d.group_stride + off;
    if (d.dtype == kOpE4M3) {  // n == 16
        const float s = d.qscale;
        uint4 w;
        w.x = pack_e4m3x4(y[0] * s, y[1] * s, y[2] * s, y[3] * s);
        w.y = pack_e4m3x4(y[4] * s, y[5] * s, y[6] * s, y[7] * s);
        w.z = pack_e4m3x4(y[8] * s, y[9] * s, y[10] * s, y[11] * s);
        w.w = pack_e4m3x4(y[12] * s, y[13] * s, y[14] * s, y[15] * s);
        *reinterpret_cast<uint4*>(o) = w;
    } else {  // 8 channels per cell; n == 8 or 16 (then two cells)
        for (int c0 = 0; c0 < n; c0 += 8)
            *reinterpret_cast<uint4*>(o + (c0 / 8) * d.group_stride) = pack_cell16(y + c0, d.dtype);
    }
}

// Block = (plane chunk, z, batch x channel group); thread = kNormVox interior voxels of one z
// plane x CPT channels (one 16-channel e4m3 cell, or one or two 8-channel f16 cells). The cells
// of all kNormVox voxels are loaded before any is used, for memory-level parallelism.
// MODE 0: any destinations (store_dest); 1: one plain e4m3 destination, the common case, the
// store reduced to one 16-byte e4m3 cell; 2: an e4m3 phase-split destination d0 plus a plain e4m3
// d1 (an encoder stage's output: the stride-2 conv's input and the decoder's skip half), both
// stores resolved at compile time; 3 and 4: the same two shapes with 16-bit destinations (a pair
// of 8-channel cells per 16 channels), for the layers that run on f16 / bf16 operands. The pass
// is bound by memory latency, not by bytes in flight per
// thread: two voxels per thread and registers for eight CTAs per SM (six for the two-destination
// forms) measured 11% faster than four voxels at three CTAs.
constexpr int kNormThreads = 256, kNormVox = 2;
template <int CPT, int MODE>
__global__ void __launch_bounds__(kNormThreads, MODE == 1 || MODE == 3 ? 8 : 6) norm_act_kernel(const uint8_t* __restrict__ pre,
                                                                         int64_t pbs, int64_t pgs, GridGeom g,
                                                                         FastDiv fw, int C,
                                                                         const float* __restrict__ ss, float slope,
                                                                         NormDest d0, NormDest d1, unsigned* amax) {
    constexpr int NC = CPT / 8;  // f16 cells per voxel
    const int ngo = C / CPT;
    const int b = blockIdx.z / ngo, go = blockIdx.z - b * ngo;
    const int gi0 = go * NC;
    const int zp = blockIdx.y + 1;
    const int Hp = g.H + 2, Wp = g.W + 2;
    const uint32_t HW = static_cast<uint32_t>(g.H) * g.W;
    __shared__ float2 s_ss[CPT];  // {scale, shift} of the block's channels
    if (threadIdx.x < CPT)
        s_ss[threadIdx.x] = __ldg(reinterpret_cast<const float2*>(ss) + static_cast<int64_t>(b) * C + gi0 * 8 +
                                  threadIdx.x);
    __syncthreads();
    const uint8_t* pb = pre + b * pbs + gi0 * pgs;
    uint4 cell[kNormVox][NC];
    int yp[kNormVox], xp[kNormVox];
    const uint32_t i0 = blockIdx.x * (kNormThreads * kNormVox) + threadIdx.x;
#pragma unroll
    for (int k = 0; k < kNormVox; ++k) {
        const uint32_t i = i0 + k * kNormThreads;
        yp[k] = -1;
        if (i < HW) {
            const uint32_t y = fdiv(i, fw);
            yp[k] = static_cast<int>(y) + 1;
            xp[k] = static_cast<int>(i - y * fw.d) + 1;
            const int64_t row = (static_cast<int64_t>(zp) * Hp + yp[k]) * Wp + xp[k];
#pragma unroll
            for (int q = 0; q < NC; ++q) cell[k][q] = __ldcs(reinterpret_cast<const uint4*>(pb + q * pgs + row * 16));
        }
    }
    float mx = 0.f;
#pragma unroll
    for (int k = 0; k < kNormVox; ++k) {
        if (yp[k] < 0) continue;
        float v[CPT];
#pragma unroll
        for (int q = 0; q < NC; ++q) {
            float f[8];
            unpack_cell16(cell[k][q], kOpF16, f);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float2 t = s_ss[q * 8 + j];
                float yv = fmaf(f[j], t.x, t.y);
                yv = yv >= 0.f ? yv : yv * slope;
                v[q * 8 + j] = yv;
                mx = fmaxf(mx, fabsf(yv));
            }
        }
        const int64_t row = (static_cast<int64_t>(zp) * Hp + yp[k]) * Wp + xp[k];
        if constexpr (MODE == 1) {
            const float qs = d0.qscale;
            uint4 w;
            w.x = pack_e4m3x4(v[0] * qs, v[1] * qs, v[2] * qs, v[3] * qs);
            w.y = pack_e4m3x4(v[4] * qs, v[5] * qs, v[6] * qs, v[7] * qs);
            w.z = pack_e4m3x4(v[8] * qs, v[9] * qs, v[10] * qs, v[11] * qs);
            w.w = pack_e4m3x4(v[12] * qs, v[13] * qs, v[14] * qs, v[15] * qs);
            *reinterpret_cast<uint4*>(d0.ptr + b * d0.batch_stride + go * d0.group_stride + row * 16) = w;
        } else if constexpr (MODE == 2) {
            const float q0 = d0.qscale, q1 = d1.qscale;
            uint4 w;
            w.x = pack_e4m3x4(v[0] * q0, v[1] * q0, v[2] * q0, v[3] * q0);
            w.y = pack_e4m3x4(v[4] * q0, v[5] * q0, v[6] * q0, v[7] * q0);
            w.z = pack_e4m3x4(v[8] * q0, v[9] * q0, v[10] * q0, v[11] * q0);
            w.w = pack_e4m3x4(v[12] * q0, v[13] * q0, v[14] * q0, v[15] * q0);
            *reinterpret_cast<uint4*>(d0.ptr + b * d0.batch_stride + go * d0.group_stride +
                                      phase_cell_offset(d0.phase, zp, yp[k], xp[k], d0.pHp, d0.pWp, d0.phase_stride)) = w;
            w.x = pack_e4m3x4(v[0] * q1, v[1] * q1, v[2] * q1, v[3] * q1);
            w.y = pack_e4m3x4(v[4] * q1, v[5] * q1, v[6] * q1, v[7] * q1);
            w.z = pack_e4m3x4(v[8] * q1, v[9] * q1, v[10] * q1, v[11] * q1);
            w.w = pack_e4m3x4(v[12] * q1, v[13] * q1, v[14] * q1, v[15] * q1);
            *reinterpret_cast<uint4*>(d1.ptr + b * d1.batch_stride + go * d1.group_stride + row * 16) = w;
        } else if constexpr (MODE == 3 || MODE == 4) {
            // 16-bit destinations (two f16 / bf16 cells per 16 channels): d0 plain (MODE 3), or d0
            // phase-split and d1 plain (MODE 4), the cell type fixed per launch by d0.dtype
            const uint4 c0 = pack_cell16(v, d0.dtype), c1 = pack_cell16(v + 8, d0.dtype);
            int64_t off0 = row * 16;
            if constexpr (MODE == 4) off0 = phase_cell_offset(d0.phase, zp, yp[k], xp[k], d0.pHp, d0.pWp, d0.phase_stride);
            uint8_t* o0 = d0.ptr + b * d0.batch_stride + gi0 * d0.group_stride + off0;
            *reinterpret_cast<uint4*>(o0) = c0;
            *reinterpret_cast<uint4*>(o0 + d0.group_stride) = c1;
            if constexpr (MODE == 4) {
                uint8_t* o1 = d1.ptr + b * d1.batch_stride + gi0 * d1.group_stride + row * 16;
                *reinterpret_cast<uint4*>(o1) = c0;
                *reinterpret_cast<uint4*>(o1 + d1.group_stride) = c1;
            }
        } else {
            store_dest(d0, b, d0.dtype == kOpE4M3 ? go : gi0, row, zp, yp[k], xp[k], v, CPT);
            store_dest(d1, b, d1.dtype == kOpE4M3 ? go : gi0, row, zp, yp[k], xp[k], v, CPT);
        }
    }
    if (amax) {
        for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if ((threadIdx.x & 31) == 0) atomicMax(amax, __float_as_uint(mx));
    }
}

// One thread = one interior voxel x 16 channels (two f16 cells of every tensor).
__global__ void __launch_bounds__(kEwThreads) block_out_kernel(BlockOut p, FastDiv fw) {
    const int ngo = p.C / 16;
    const int b = blockIdx.z / ngo, go = blockIdx.z - b * ngo;
    const int zp = blockIdx.y + 1;
    const uint32_t HW = static_cast<uint32_t>(p.g.H) * p.g.W;
    const uint32_t i = blockIdx.x * kEwThreads + threadIdx.x;
    __shared__ float s_ss[16][2], s_rs[16][2], s_cg[16];
    if (threadIdx.x < 16) {
        const int c = go * 16 + threadIdx.x;
        const float2 t = __ldg(reinterpret_cast<const float2*>(p.ss) + static_cast<int64_t>(b) * p.C + c);
        s_ss[threadIdx.x][0] = t.x;
        s_ss[threadIdx.x][1] = t.y;
        const float2 r = p.res_ss ? __ldg(reinterpret_cast<const float2*>(p.res_ss) + static_cast<int64_t>(b) * p.C + c)
                                  : make_float2(1.f, 0.f);
        s_rs[threadIdx.x][0] = r.x;
        s_rs[threadIdx.x][1] = r.y;
        s_cg[threadIdx.x] = p.cgate ? __ldg(p.cgate + c) : 1.f;
    }
    __syncthreads();
    if (i >= HW) return;
    const uint32_t y = fdiv(i, fw);
    const int yp = static_cast<int>(y) + 1, xp = static_cast<int>(i - y * fw.d) + 1;
    const int Hp = p.g.H + 2, Wp = p.g.W + 2;
    const int64_t row = (static_cast<int64_t>(zp) * Hp + yp) * Wp + xp;
    const float sg = p.sgate ? __ldg(p.sgate + ((static_cast<int64_t>(b) * p.g.D + (zp - 1)) * p.g.H + y) * p.g.W +
                                     (xp - 1))
                             : 0.f;
    float v[16];
    float mx = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int gi = go * 2 + h;
        float o[8], r[8];
        unpack_cell16(__ldcs(reinterpret_cast<const uint4*>(p.pre + b * p.pre_bs + gi * p.pre_gs + row * 16)), kOpF16,
                      o);
        unpack_cell16(__ldcs(reinterpret_cast<const uint4*>(p.res + b * p.res_bs + gi * p.res_gs + row * 16)), kOpF16,
                      r);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = h * 8 + j;
            const float out = fmaf(o[j], s_ss[c][0], s_ss[c][1]);
            const float res = fmaf(r[j], s_rs[c][0], s_rs[c][1]);
            float t = fmaf(out, s_cg[c] + sg, res);
            t = t >= 0.f ? t : t * p.slope;
            v[c] = t;
            mx = fmaxf(mx, fabsf(t));
        }
    }
#pragma unroll
    for (int k = 0; k < 3; ++k)
        store_dest(p.d[k], b, p.d[k].dtype == kOpE4M3 ? go : go * 2, row, zp, yp, xp, v, 16);
    if (p.amax) {
        for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if ((threadIdx.x & 31) == 0) atomicMax(p.amax, __float_as_uint(mx));
    }
}

// One thread = one interior voxel: a dot product over all C channels of the normalised tensor.
__global__ void __launch_bounds__(kEwThreads) sse_gate_kernel(const uint8_t* __restrict__ pre, int64_t pbs,
                                                               int64_t pgs, const float* __restrict__ ss,
                                                               const float* __restrict__ w, float bias, GridGeom g,
                                                               int C, FastDiv fw, float* __restrict__ sgate) {
    const int b = blockIdx.z, z = blockIdx.y;
    extern __shared__ float s_coef[];  // [C][2]: w * scale, w * shift
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float2 t = __ldg(reinterpret_cast<const float2*>(ss) + static_cast<int64_t>(b) * C + c);
        s_coef[2 * c] = w[c] * t.x;
        s_coef[2 * c + 1] = w[c] * t.y;
    }
    __syncthreads();
    const uint32_t HW = static_cast<uint32_t>(g.H) * g.W;
    const uint32_t i = blockIdx.x * kEwThreads + threadIdx.x;
    if (i >= HW) return;
    const uint32_t y = fdiv(i, fw);
    const int x = static_cast<int>(i - y * fw.d);
    const int64_t row = (static_cast<int64_t>(z + 1) * (g.H + 2) + y + 1) * (g.W + 2) + x + 1;
    float acc = bias;
    for (int gi = 0; gi < C / 8; ++gi) {
        float f[8];
        unpack_cell16(__ldg(reinterpret_cast<const uint4*>(pre + b * pbs + gi * pgs + row * 16)), kOpF16, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(f[j], s_coef[2 * (gi * 8 + j)], acc + s_coef[2 * (gi * 8 + j) + 1]);
    }
    sgate[((static_cast<int64_t>(b) * g.D + z) * g.H + y) * g.W + x] = 1.f / (1.f + expf(-acc));
}

// One thread = one output voxel x one 8-channel f16 group.
__global__ void __launch_bounds__(kEwThreads) avgpool2_f16_kernel(const uint8_t* __restrict__ src, int64_t sbs,
                                                                   int64_t sgs, GridGeom gin, uint8_t* dst,
                                                                   int64_t dbs, int64_t dgs, int groups,
                                                                   FastDiv fw) {
    const int bg = blockIdx.z, b = bg / groups, gi = bg - b * groups, z = blockIdx.y;
    const int Ho = gin.H / 2, Wo = gin.W / 2;
    const uint32_t i = blockIdx.x * kEwThreads + threadIdx.x;
    if (i >= static_cast<uint32_t>(Ho) * Wo) return;
    const uint32_t y = fdiv(i, fw);
    const int x = static_cast<int>(i - y * fw.d);
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const uint8_t* sb = src + b * sbs + gi * sgs;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int zz = 2 * z + (k >> 2), yy = 2 * static_cast<int>(y) + ((k >> 1) & 1), xx = 2 * x + (k & 1);
        const int64_t row = (static_cast<int64_t>(zz + 1) * (gin.H + 2) + yy + 1) * (gin.W + 2) + xx + 1;
        float f[8];
        unpack_cell16(__ldg(reinterpret_cast<const uint4*>(sb + row * 16)), kOpF16, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] += f[j];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] *= 0.125f;
    const int64_t orow = (static_cast<int64_t>(z + 1) * (Ho + 2) + y + 1) * (Wo + 2) + x + 1;
    *reinterpret_cast<uint4*>(dst + b * dbs + gi * dgs + orow * 16) = pack_cell16(a, kOpF16);
}

__constant__ float c_head_w[2 * 64];
__constant__ float c_head_b[2];

// Block = (plane chunk, z, batch item); thread = one voxel. Scale/shift of the batch item's C
// channels sit in shared memory, the head weights in constant memory.
// One thread per tile voxel, five 256-thread CTAs per SM (48 registers, no spill). The thread's
// pre-norm cells are requested before the block's {scale, shift} table is loaded, so the two
// latencies overlap (a block lives for one voxel per thread).
__global__ void __launch_bounds__(kEwThreads, 5) head_blend_kernel(HeadParams h, FastDiv fp) {
    const int Hp = h.Py + 2, Wp = h.Px + 2;
    const int b = blockIdx.z, z = blockIdx.y;
    __shared__ float2 s_ss[64];
    const uint32_t i = blockIdx.x * kEwThreads + threadIdx.x;
    const bool live = i < static_cast<uint32_t>(h.Py) * h.Px;
    const int G = h.C / 8;
    int y = 0, x = 0;
    uint4 cells[8];
    if (live) {
        y = static_cast<int>(fdiv(i, fp));
        x = static_cast<int>(i - static_cast<uint32_t>(y) * h.Px);
        const int64_t row = (static_cast<int64_t>(z + 1) * Hp + (y + 1)) * Wp + (x + 1);
        const uint8_t* pb = h.pre + b * h.pre_batch_stride + row * 16;
#pragma unroll
        for (int gi = 0; gi < 8; ++gi)
            if (gi < G) cells[gi] = __ldcs(reinterpret_cast<const uint4*>(pb + gi * h.pre_group_stride));
    }
    if (threadIdx.x < h.C)
        s_ss[threadIdx.x] = __ldg(reinterpret_cast<const float2*>(h.ss) + static_cast<int64_t>(b) * h.C + threadIdx.x);
    __syncthreads();
    if (!live) return;
    float l0 = c_head_b[0], l1 = h.ncls > 1 ? c_head_b[1] : 0.f;
#pragma unroll
    for (int gi = 0; gi < 8; ++gi) {
        if (gi >= G) break;
        float f[8];
        unpack_cell16(cells[gi], kOpF16, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = gi * 8 + j;
            const float2 sc = s_ss[c];
            float yv = fmaf(f[j], sc.x, sc.y);
            yv = yv >= 0.f ? yv : yv * h.slope;
            l0 = fmaf(c_head_w[c], yv, l0);
            if (h.ncls > 1) l1 = fmaf(c_head_w[h.C + c], yv, l1);
        }
    }
    float p;
    if (h.sigmoid) {
        p = 1.f / (1.f + expf(-l0));
    } else {
        const float m = fmaxf(l0, l1);
        const float e0 = expf(l0 - m), e1 = expf(l1 - m);
        p = (h.channel == 1 ? e1 : e0) / (e0 + e1);
    }
    if (isnan(p)) p = 0.f;
    else if (isinf(p)) p = p > 0.f ? 1.f : 0.f;
    const int64_t n = static_cast<int64_t>(h.Pz) * h.Py * h.Px;
    int sz = z, sy = y, sx = x;  // tile voxel this output belongs to (its TTA member's source; cubes)
    if (h.tta) {
        tta_source(h.tta[b], h.Px, z, y, x, sz, sy, sx);
        p *= h.tta_scale;
    }
    if (h.prob) h.prob[b * n + (static_cast<int64_t>(sz) * h.Py + sy) * h.Px + sx] = p;
    if (h.acc) {
        const TileOrigin t = h.tiles[b];
        const int z = sz, y = sy, x = sx;
        const int64_t oz = t.z0 + z, oy = t.y0 + y, ox = t.x0 + x;
        const int64_t az = oz + h.acc_z_shift;
        const bool crop = h.acc_dy > 0;
        const int64_t ay = crop ? oy + h.acc_y_shift : oy, ax = crop ? ox + h.acc_x_shift : ox;
        const int64_t ady = crop ? h.acc_dy : h.dy, adx = crop ? h.acc_dx : h.dx;
        if (oz < h.dz && oy < h.dy && ox < h.dx && az >= 0 && az < h.acc_dz && ay >= 0 && ay < ady && ax >= 0 &&
            ax < adx) {
            // (gz*gy)*gx*p in the reference's order (src/ml/infer.hpp:631-653)
            const float wzy = __fmul_rn(__ldg(h.gz + z), __ldg(h.gy + y));
            const float c = __fmul_rn(__fmul_rn(wzy, __ldg(h.gx + x)), p);
            atomicAdd(h.acc + (az * ady + ay) * adx + ax, c);
        }
    }
}

__global__ void __launch_bounds__(kEwThreads) scatter_tile_kernel(const float* __restrict__ prob, int P, int64_t z0,
                                                                   int64_t y0, int64_t x0, int64_t dz, int64_t dy,
                                                                   int64_t dx, int64_t z_floor,
                                                                   const float* __restrict__ gauss, float* acc,
                                                                   int64_t acc_z_shift, int64_t acc_dz, FastDiv fp) {
    const int z = blockIdx.y;
    const uint32_t i = blockIdx.x * kEwThreads + threadIdx.x;
    if (i >= static_cast<uint32_t>(P) * P) return;
    const int y = static_cast<int>(fdiv(i, fp));
    const int x = static_cast<int>(i - static_cast<uint32_t>(y) * P);
    const int64_t oz = z0 + z, oy = y0 + y, ox = x0 + x;
    const int64_t az = oz + acc_z_shift;
    if (oz < 0 || oz >= dz || oy < 0 || oy >= dy || ox < 0 || ox >= dx || oz < z_floor || az < 0 || az >= acc_dz)
        return;
    const float p = __ldg(prob + static_cast<int64_t>(z) * P * P + i);
    // (gz*gy)*gx*p in the reference's order (src/ml/global_accum.hpp:103-111)
    const float wzy = __fmul_rn(__ldg(gauss + z), __ldg(gauss + y));
    atomicAdd(acc + (az * dy + oy) * dx + ox, __fmul_rn(__fmul_rn(wzy, __ldg(gauss + x)), p));
}

// acc and prob may alias when z_begin == 0 (in-place normalise): each element is read before it
// is written, by the same thread.
__global__ void accum_finalize_kernel(const float* acc, int64_t dz, int64_t dy, int64_t dx,
                                      int64_t z_begin, int64_t z_end, const float* __restrict__ Wz,
                                      const float* __restrict__ Wy, const float* __restrict__ Wx, float* prob,
                                      uint8_t* __restrict__ u8) {
    const int64_t plane = dy * dx;
    const int64_t total = (z_end - z_begin) * plane;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t z = z_begin + i / plane;
        const int64_t r = i % plane;
        const int64_t y = r / dx, x = r % dx;
        const int64_t idx = z * plane + r;  // accumulator index
        const int64_t oidx = i;               // output index: plane z_begin is output plane 0
        // w = (Wz*Wy)*Wx; v /= w when w > 0 (src/ml/infer.hpp:510-521)
        const float w = __fmul_rn(__fmul_rn(__ldg(Wz + z), __ldg(Wy + y)), __ldg(Wx + x));
        float v = acc[idx];
        if (w > 0.f) v = __fdiv_rn(v, w);
        if (prob) prob[oidx] = v;
        if (u8) {
            const float c = fminf(fmaxf(v, 0.f), 1.f);
            // (u8)(clamp(v,0,1)*255+0.5) (src/ml/inference.cpp:343-351)
            u8[oidx] = static_cast<uint8_t>(__fadd_rn(__fmul_rn(c, 255.f), 0.5f));
        }
    }
}

__global__ void accum_add_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t n) {
    const int64_t n4 = n / 4;
    float4* d4 = reinterpret_cast<float4*>(dst);
    const float4* s4 = reinterpret_cast<const float4*>(src);
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float4 a = d4[i];
        const float4 b = s4[i];
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
        d4[i] = a;
    }
    for (int64_t i = n4 * 4 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] += src[i];
}

__global__ void accum_add_scalar_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] += src[i];
}

int grid_for(int64_t n, int threads) {
    int64_t g = (n + threads - 1) / threads;
    if (g > 148 * 16) g = 148 * 16;
    if (g < 1) g = 1;
    return static_cast<int>(g);
}

}  // namespace

cudaError_t launch_tile_sums(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, const TileOrigin* tiles,
                             int ntiles, TileDims P, unsigned long long* sums, cudaStream_t s, unsigned* hist) {
    if (ntiles < 1 || ntiles > 65535 || P.z < 1 || P.y < 1 || P.x < 1) return cudaErrorInvalidValue;
    const int64_t lines = static_cast<int64_t>(P.z) * P.y;
    const int gx = grid_for(lines, (kEwThreads / 32) * 4);  // four lines per warp
    count_launch();
    if (hist)
        tile_sums_kernel<true><<<dim3(gx, ntiles), kEwThreads, 0, s>>>(vol, dz, dy, dx, tiles, P, sums, hist);
    else
        tile_sums_kernel<false><<<dim3(gx, ntiles), kEwThreads, 0, s>>>(vol, dz, dy, dx, tiles, P, sums, nullptr);
    return cudaGetLastError();
}

cudaError_t launch_tile_lut(const unsigned long long* sums, const unsigned* hist, int ntiles, int64_t n, int norm,
                            float* luts, uint8_t* const_flag, cudaStream_t s) {
    if (ntiles < 1 || norm < 0 || norm > 2 || (norm == 1 && !hist)) return cudaErrorInvalidValue;
    count_launch();
    tile_lut_kernel<<<ntiles, 256, 0, s>>>(sums, hist, n, norm, luts, const_flag);
    return cudaGetLastError();
}

cudaError_t launch_tile_norm(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, const TileOrigin* tiles,
                             int ntiles, TileDims P, const unsigned long long* sums, uint8_t* l0, int64_t l0_batch_stride,
                             int64_t l0_group_stride, int l0_type, float* f32_out, cudaStream_t s, const uint8_t* tta,
                             const float* luts) {
    if (ntiles < 1 || ntiles > 65535 || P.z < 1 || P.y < 1 || P.x < 1) return cudaErrorInvalidValue;
    if (tta && !(P.z == P.y && P.y == P.x)) return cudaErrorInvalidValue;  // the symmetries permute axes
    const int64_t lines = static_cast<int64_t>(P.z) * P.y;
    const int gx = grid_for(lines, (kEwThreads / 32) * 2);  // two lines per warp
    count_launch();
    tile_norm_kernel<<<dim3(gx, ntiles), kEwThreads, 0, s>>>(vol, dz, dy, dx, tiles, P, sums, luts, l0,
                                                             l0_batch_stride, l0_group_stride, l0_type, f32_out, tta);
    return cudaGetLastError();
}

// about 64 records per slice (eight per warp, loads batched four deep), at most kMaxStatSlices
// slices: more slices add blocks but lengthen the last block's serial walk over them
int in_stats_slices(int nrec) { return nrec < 128 ? 1 : (nrec / 64 < kMaxStatSlices ? nrec / 64 : kMaxStatSlices); }

cudaError_t launch_in_finalize(float* partials, int B, int nrec, int C, double count, const float* gamma,
                               const float* beta, const float* ratio, float eps, double* work, unsigned* done,
                               float* ss, cudaStream_t s) {
    if (nrec < 1 || C < 1 || B < 1) return cudaErrorInvalidValue;
    const int S = in_stats_slices(nrec);
    count_launch();
    in_stats_kernel<<<dim3((C + 31) / 32, B, S), 256, 0, s>>>(partials, nrec, C, S, count, gamma, beta, ratio, eps,
                                                             work, done, ss);
    return cudaGetLastError();
}

cudaError_t launch_norm_act(const uint8_t* pre, int64_t pbs, int64_t pgs, GridGeom g, int C, int B, const float* ss,
                            float slope, NormDest d0, NormDest d1, unsigned* amax, cudaStream_t s) {
    const bool any_fp8 = (d0.ptr && d0.dtype == kOpE4M3) || (d1.ptr && d1.dtype == kOpE4M3);
    const int cpt = (any_fp8 || C % 16 == 0) ? 16 : 8;
    if (C % cpt || static_cast<int64_t>(g.H) * g.W >= (1ll << 31) || g.D > 65535 || B * (C / cpt) > 65535)
        return cudaErrorInvalidValue;
    const uint32_t HW = static_cast<uint32_t>(g.H) * g.W;
    const dim3 grid((HW + kNormThreads * kNormVox - 1) / (kNormThreads * kNormVox), g.D, B * (C / cpt));
    const FastDiv fw = make_fastdiv(static_cast<uint32_t>(g.W));
    count_launch();
    const bool e4 = cpt == 16 && d0.ptr && d0.dtype == kOpE4M3 && !d0.phase && !d1.ptr;
    // one e4m3 phase-split destination and one plain e4m3 destination, in either order (the two
    // stores are independent): the phase-split one goes first
    const bool pair = cpt == 16 && d0.ptr && d1.ptr && d0.dtype == kOpE4M3 && d1.dtype == kOpE4M3 &&
                      (d0.phase != 0) != (d1.phase != 0);
    // 16-bit destinations of one type: one plain cell pair, or a phase-split copy + a plain copy
    const bool h0 = cpt == 16 && d0.ptr && d0.dtype != kOpE4M3;
    const bool h_one = h0 && !d0.phase && !d1.ptr;
    const bool h_pair = h0 && d1.ptr && d1.dtype == d0.dtype && (d0.phase != 0) != (d1.phase != 0);
    if (h_one)
        norm_act_kernel<16, 3><<<grid, kNormThreads, 0, s>>>(pre, pbs, pgs, g, fw, C, ss, slope, d0, d1, amax);
    else if (h_pair && d0.phase)
        norm_act_kernel<16, 4><<<grid, kNormThreads, 0, s>>>(pre, pbs, pgs, g, fw, C, ss, slope, d0, d1, amax);
    else if (h_pair)
        norm_act_kernel<16, 4><<<grid, kNormThreads, 0, s>>>(pre, pbs, pgs, g, fw, C, ss, slope, d1, d0, amax);
    else if (e4)
        norm_act_kernel<16, 1><<<grid, kNormThreads, 0, s>>>(pre, pbs, pgs, g, fw, C, ss, slope, d0, d1, amax);
    else if (pair && d0.phase)
        norm_act_kernel<16, 2><<<grid, kNormThreads, 0, s>>>(pre, pbs, pgs, g, fw, C, ss, slope, d0, d1, amax);
    else if (pair)
        norm_act_kernel<16, 2><<<grid, kNormThreads, 0, s>>>(pre, pbs, pgs, g, fw, C, ss, slope, d1, d0, amax);
    else if (cpt == 16)
        norm_act_kernel<16, 0><<<grid, kNormThreads, 0, s>>>(pre, pbs, pgs, g, fw, C, ss, slope, d0, d1, amax);
    else
        norm_act_kernel<8, 0><<<grid, kNormThreads, 0, s>>>(pre, pbs, pgs, g, fw, C, ss, slope, d0, d1, amax);
    return cudaGetLastError();
}

cudaError_t launch_block_out(const BlockOut& p, cudaStream_t s) {
    if (p.C % 16 || !p.pre || !p.ss || !p.res || p.g.D > 65535 || p.B * (p.C / 16) > 65535) return cudaErrorInvalidValue;
    const uint32_t HW = static_cast<uint32_t>(p.g.H) * p.g.W;
    count_launch();
    block_out_kernel<<<dim3((HW + kEwThreads - 1) / kEwThreads, p.g.D, p.B * (p.C / 16)), kEwThreads, 0, s>>>(
        p, make_fastdiv(static_cast<uint32_t>(p.g.W)));
    return cudaGetLastError();
}

cudaError_t launch_sse_gate(const uint8_t* pre, int64_t pre_bs, int64_t pre_gs, const float* ss, const float* w,
                            float bias, GridGeom g, int C, int B, float* sgate, cudaStream_t s) {
    if (C % 8 || C > 4096 || g.D > 65535 || B > 65535) return cudaErrorInvalidValue;
    const uint32_t HW = static_cast<uint32_t>(g.H) * g.W;
    count_launch();
    sse_gate_kernel<<<dim3((HW + kEwThreads - 1) / kEwThreads, g.D, B), kEwThreads, sizeof(float) * 2 * C, s>>>(
        pre, pre_bs, pre_gs, ss, w, bias, g, C, make_fastdiv(static_cast<uint32_t>(g.W)), sgate);
    return cudaGetLastError();
}

cudaError_t launch_avgpool2_f16(const uint8_t* src, int64_t src_bs, int64_t src_gs, GridGeom gin, uint8_t* dst,
                                int64_t dst_bs, int64_t dst_gs, int groups, int B, cudaStream_t s) {
    if (gin.D % 2 || gin.H % 2 || gin.W % 2 || B * groups > 65535) return cudaErrorInvalidValue;
    const uint32_t HW = static_cast<uint32_t>(gin.H / 2) * (gin.W / 2);
    count_launch();
    avgpool2_f16_kernel<<<dim3((HW + kEwThreads - 1) / kEwThreads, gin.D / 2, B * groups), kEwThreads, 0, s>>>(
        src, src_bs, src_gs, gin, dst, dst_bs, dst_gs, groups, make_fastdiv(static_cast<uint32_t>(gin.W / 2)));
    return cudaGetLastError();
}

cudaError_t launch_head_blend(const HeadParams& h, cudaStream_t s) {
    if (h.ncls < 1 || h.ncls > 2 || h.C > 64 || h.C % 8 || h.B > 65535 || h.Pz < 1 || h.Pz > 65535 ||
        static_cast<int64_t>(h.Py) * h.Px >= (1ll << 31) || (h.tta && !(h.Pz == h.Py && h.Py == h.Px)))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaMemcpyToSymbolAsync(c_head_w, h.wh, sizeof(float) * h.ncls * h.C, 0,
                                            cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return e;
    e = cudaMemcpyToSymbolAsync(c_head_b, h.bh, sizeof(float) * h.ncls, 0, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return e;
    const uint32_t PP = static_cast<uint32_t>(h.Py) * h.Px;
    count_launch();
    head_blend_kernel<<<dim3((PP + kEwThreads - 1) / kEwThreads, h.Pz, h.B), kEwThreads, 0, s>>>(
        h, make_fastdiv(static_cast<uint32_t>(h.Px)));
    return cudaGetLastError();
}

cudaError_t launch_scatter_tile(const float* prob, int P, int64_t z0, int64_t y0, int64_t x0, int64_t dz, int64_t dy,
                                int64_t dx, int64_t z_floor, const float* gauss, float* acc, int64_t acc_z_shift,
                                int64_t acc_dz, cudaStream_t s) {
    if (P < 1 || P > 46340 || !prob || !gauss || !acc) return cudaErrorInvalidValue;
    const uint32_t PP = static_cast<uint32_t>(P) * P;
    count_launch();
    scatter_tile_kernel<<<dim3((PP + kEwThreads - 1) / kEwThreads, P), kEwThreads, 0, s>>>(
        prob, P, z0, y0, x0, dz, dy, dx, z_floor, gauss, acc, acc_z_shift, acc_dz, make_fastdiv(static_cast<uint32_t>(P)));
    return cudaGetLastError();
}

cudaError_t launch_accum_finalize(const float* acc, int64_t dz, int64_t dy, int64_t dx, int64_t z_begin,
                                  int64_t z_end, const float* Wz, const float* Wy, const float* Wx, float* prob,
                                  uint8_t* u8, cudaStream_t s) {
    const int64_t n = (z_end - z_begin) * dy * dx;
    if (n <= 0) return cudaSuccess;
    count_launch();
    accum_finalize_kernel<<<grid_for(n, kEwThreads), kEwThreads, 0, s>>>(acc, dz, dy, dx, z_begin, z_end, Wz, Wy,
                                                                         Wx, prob, u8);
    return cudaGetLastError();
}

cudaError_t launch_zero(void* p, size_t bytes, cudaStream_t s) { return cudaMemsetAsync(p, 0, bytes, s); }

// Agreement of two probability maps: stats[0] += #(a >= 0.5), stats[1] += #(b >= 0.5),
// stats[2] += #(both), and max |a - b| into *maxabs (float bits, both non-negative floats compare as
// unsigned). Used to choose an fp8 net's precision schedule against its 16-bit forward.
__global__ void prob_compare_kernel(const float* __restrict__ a, const float* __restrict__ b, int64_t n,
                                    unsigned long long* stats, unsigned* maxabs) {
    unsigned long long ca = 0, cb = 0, cab = 0;
    float m = 0.f;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float x = a[i], y = b[i];
        const bool pa = x >= 0.5f, pb = y >= 0.5f;
        ca += pa;
        cb += pb;
        cab += pa && pb;
        m = fmaxf(m, fabsf(x - y));
    }
    for (int o = 16; o; o >>= 1) {
        ca += __shfl_xor_sync(0xffffffffu, ca, o);
        cb += __shfl_xor_sync(0xffffffffu, cb, o);
        cab += __shfl_xor_sync(0xffffffffu, cab, o);
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    }
    if ((threadIdx.x & 31) == 0) {
        atomicAdd(stats, ca);
        atomicAdd(stats + 1, cb);
        atomicAdd(stats + 2, cab);
        atomicMax(maxabs, __float_as_uint(m));
    }
}

cudaError_t launch_prob_compare(const float* a, const float* b, int64_t n, unsigned long long* stats,
                                unsigned* maxabs, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    count_launch();
    prob_compare_kernel<<<grid_for(n, kEwThreads), kEwThreads, 0, s>>>(a, b, n, stats, maxabs);
    return cudaGetLastError();
}

cudaError_t launch_accum_add(float* dst, const float* src, int64_t n, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    count_launch();
    if ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15)  // e.g. an odd plane size
        accum_add_scalar_kernel<<<grid_for(n, kEwThreads), kEwThreads, 0, s>>>(dst, src, n);
    else
        accum_add_kernel<<<grid_for(n / 4 + 1, kEwThreads), kEwThreads, 0, s>>>(dst, src, n);
    return cudaGetLastError();
}


namespace {
__global__ void acc_max_kernel(const float* __restrict__ acc, int64_t n, unsigned* max_bits) {
    float m = 0.f;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        m = fmaxf(m, acc[i]);
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0 && m > 0.f) atomicMax(max_bits, __float_as_uint(m));
}

__global__ void acc_quant_u16_kernel(const float* __restrict__ acc, int64_t n, float inv, uint16_t* __restrict__ q) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        q[i] = static_cast<uint16_t>(__fadd_rn(__fmul_rn(acc[i], inv), 0.5f));
}
}  // namespace

cudaError_t launch_acc_max(const float* acc, int64_t n, unsigned* max_bits, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    count_launch();
    acc_max_kernel<<<static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 16)), 256, 0, s>>>(acc, n, max_bits);
    return cudaGetLastError();
}

cudaError_t launch_acc_quant_u16(const float* acc, int64_t n, float inv, uint16_t* q, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    count_launch();
    acc_quant_u16_kernel<<<static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 16)), 256, 0, s>>>(acc, n, inv, q);
    return cudaGetLastError();
}

}  // namespace fxk
