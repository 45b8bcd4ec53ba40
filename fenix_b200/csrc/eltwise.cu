// eltwise.cu — HBM-bound kernels of the inference path (see eltwise.cuh).
#include "eltwise.cuh"
#include "counters.hpp"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp8.h>

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

__global__ void tile_sums_kernel(const uint8_t* __restrict__ vol, int64_t dz, int64_t dy, int64_t dx,
                                 const TileOrigin* __restrict__ tiles, int P, unsigned long long* sums) {
    const int b = blockIdx.y;
    const TileOrigin t = tiles[b];
    const int64_t n = static_cast<int64_t>(P) * P * P;
    const bool inside = t.z0 + P <= dz && t.y0 + P <= dy && t.x0 + P <= dx;
    unsigned long long s1 = 0, s2 = 0;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int x = static_cast<int>(i % P);
        const int64_t zy = i / P;
        const int y = static_cast<int>(zy % P);
        const int z = static_cast<int>(zy / P);
        const uint32_t v = inside ? __ldg(vol + ((t.z0 + z) * dy + (t.y0 + y)) * dx + (t.x0 + x))
                                  : vol_at(vol, dz, dy, dx, t.z0 + z, t.y0 + y, t.x0 + x);
        s1 += v;
        s2 += v * v;
    }
    for (int o = 16; o >= 1; o >>= 1) {
        s1 += __shfl_down_sync(0xffffffffu, s1, o);
        s2 += __shfl_down_sync(0xffffffffu, s2, o);
    }
    __shared__ unsigned long long r1[kEwThreads / 32], r2[kEwThreads / 32];
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        r1[w] = s1;
        r2[w] = s2;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long a = 0, c = 0;
        for (int i = 0; i < kEwThreads / 32; ++i) {
            a += r1[i];
            c += r2[i];
        }
        atomicAdd(&sums[2 * b], a);
        atomicAdd(&sums[2 * b + 1], c);
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

__global__ void tile_norm_kernel(const uint8_t* __restrict__ vol, int64_t dz, int64_t dy, int64_t dx,
                                 const TileOrigin* __restrict__ tiles, int P,
                                 const unsigned long long* __restrict__ sums, uint8_t* __restrict__ l0,
                                 int64_t l0_batch_stride, int l0_type, float* __restrict__ f32_out) {
    const int b = blockIdx.y;
    __shared__ float lut[256];
    const int64_t n = static_cast<int64_t>(P) * P * P;
    build_lut(lut, sums[2 * b], sums[2 * b + 1], n);
    __syncthreads();
    const TileOrigin t = tiles[b];
    const int Pp = P + 2;
    const bool inside = t.z0 + P <= dz && t.y0 + P <= dy && t.x0 + P <= dx;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int x = static_cast<int>(i % P);
        const int64_t zy = i / P;
        const int y = static_cast<int>(zy % P);
        const int z = static_cast<int>(zy / P);
        float v[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int xx = x - 1 + k;
            if (xx < 0 || xx >= P) {
                v[k] = 0.f;
            } else {
                const uint8_t u = inside ? __ldg(vol + ((t.z0 + z) * dy + (t.y0 + y)) * dx + (t.x0 + xx))
                                         : vol_at(vol, dz, dy, dx, t.z0 + z, t.y0 + y, t.x0 + xx);
                v[k] = lut[u];
            }
        }
        const int64_t row = (static_cast<int64_t>(z + 1) * Pp + (y + 1)) * Pp + (x + 1);
        if (l0) {
            const float cell[8] = {v[0], v[1], v[2], 0.f, 0.f, 0.f, 0.f, 0.f};
            *reinterpret_cast<uint4*>(l0 + b * l0_batch_stride + row * 16) = pack_cell16(cell, l0_type);
        }
        if (f32_out) f32_out[b * n + i] = v[1];
    }
}

__global__ void in_finalize_kernel(const float* __restrict__ partials, int nrec, int C, double count,
                                   const float* __restrict__ gamma, const float* __restrict__ beta, float eps,
                                   float* __restrict__ ss) {
    // block: 32 channels x 32 record slices
    const int b = blockIdx.y;
    const int lane = threadIdx.x & 31;
    const int slice = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    double a1 = 0.0, a2 = 0.0;
    if (c < C) {
        const float* base = partials + static_cast<int64_t>(b) * nrec * C * 2;
        for (int r = slice; r < nrec; r += 32) {
            const float2 v = *reinterpret_cast<const float2*>(base + (static_cast<int64_t>(r) * C + c) * 2);
            a1 += v.x;
            a2 += v.y;
        }
    }
    __shared__ double s1[32][33], s2[32][33];
    s1[slice][lane] = a1;
    s2[slice][lane] = a2;
    __syncthreads();
    if (slice == 0 && c < C) {
        double t1 = 0.0, t2 = 0.0;
        for (int i = 0; i < 32; ++i) {
            t1 += s1[i][lane];
            t2 += s2[i][lane];
        }
        const double mean = t1 / count;
        double var = t2 / count - mean * mean;
        if (var < 0.0) var = 0.0;
        const double rstd = 1.0 / sqrt(var + static_cast<double>(eps));
        const double sc = static_cast<double>(gamma ? gamma[c] : 1.f) * rstd;
        const double sh = static_cast<double>(beta ? beta[c] : 0.f) - mean * sc;
        ss[(static_cast<int64_t>(b) * C + c) * 2 + 0] = static_cast<float>(sc);
        ss[(static_cast<int64_t>(b) * C + c) * 2 + 1] = static_cast<float>(sh);
    }
}


__device__ __forceinline__ void store_dest(const NormDest& d, int b, int gout, int64_t row, int zp, int yp, int xp,
                                           const float* y, int n) {
    if (!d.ptr) return;
    int64_t off;
    if (d.phase) {
        const int phi = ((zp & 1) << 2) | ((yp & 1) << 1) | (xp & 1);
        const int64_t prow = (static_cast<int64_t>(zp >> 1) * d.pHp + (yp >> 1)) * d.pWp + (xp >> 1);
        off = phi * d.phase_stride + prow * 16;
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

// One thread = one interior voxel x one 16-channel pair of bf16 pre-norm cells (or the single
// 8-channel cell when C is not a multiple of 16).
__global__ void norm_act_kernel(const uint8_t* __restrict__ pre, int64_t pbs, int64_t pgs, GridGeom g, int C,
                                int B, const float* __restrict__ ss, float slope, NormDest d0, NormDest d1,
                                unsigned* amax, int cpt) {
    const int Hp = g.H + 2, Wp = g.W + 2;
    const int64_t vox = static_cast<int64_t>(g.D) * g.H * g.W;
    const int ngo = C / cpt;
    const int64_t total = vox * ngo * B;
    float mx = 0.f;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int x = static_cast<int>(i % g.W);
        int64_t t = i / g.W;
        const int y = static_cast<int>(t % g.H);
        t /= g.H;
        const int z = static_cast<int>(t % g.D);
        t /= g.D;
        const int go = static_cast<int>(t % ngo);
        const int b = static_cast<int>(t / ngo);
        const int zp = z + 1, yp = y + 1, xp = x + 1;
        const int64_t row = (static_cast<int64_t>(zp) * Hp + yp) * Wp + xp;
        float v[16];
        const int gi0 = go * cpt / 8;
        for (int k = 0; k < cpt / 8; ++k) {
            const uint4 w = *reinterpret_cast<const uint4*>(pre + b * pbs + (gi0 + k) * pgs + row * 16);
            float f[8];
            unpack_cell16(w, kOpF16, f);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = (gi0 + k) * 8 + j;
                const float2 sc = *reinterpret_cast<const float2*>(ss + (static_cast<int64_t>(b) * C + c) * 2);
                float yv = fmaf(f[j], sc.x, sc.y);
                yv = yv >= 0.f ? yv : yv * slope;
                v[k * 8 + j] = yv;
                mx = fmaxf(mx, fabsf(yv));
            }
        }
        store_dest(d0, b, d0.dtype == kOpE4M3 ? go : gi0, row, zp, yp, xp, v, cpt);
        store_dest(d1, b, d1.dtype == kOpE4M3 ? go : gi0, row, zp, yp, xp, v, cpt);
    }
    if (amax) {
        for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if ((threadIdx.x & 31) == 0) atomicMax(amax, __float_as_uint(mx));
    }
}

__constant__ float c_head_w[2 * 64];
__constant__ float c_head_b[2];

__global__ void head_blend_kernel(HeadParams h) {
    const int P = h.P, Pp = P + 2;
    const int64_t n = static_cast<int64_t>(P) * P * P;
    const int G = h.C / 8;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n * h.B;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int b = static_cast<int>(i / n);
        const int64_t li = i - b * n;
        const int x = static_cast<int>(li % P);
        const int y = static_cast<int>((li / P) % P);
        const int z = static_cast<int>(li / (static_cast<int64_t>(P) * P));
        const int64_t row = (static_cast<int64_t>(z + 1) * Pp + (y + 1)) * Pp + (x + 1);
        float l0 = c_head_b[0], l1 = h.ncls > 1 ? c_head_b[1] : 0.f;
        for (int gi = 0; gi < G; ++gi) {
            const uint4 w = *reinterpret_cast<const uint4*>(h.pre + b * h.pre_batch_stride + gi * h.pre_group_stride +
                                                            row * 16);
            float f[8];
            unpack_cell16(w, kOpF16, f);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = gi * 8 + j;
                const float2 sc = *reinterpret_cast<const float2*>(h.ss + (static_cast<int64_t>(b) * h.C + c) * 2);
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
        if (h.prob) h.prob[i] = p;
        if (h.acc) {
            const TileOrigin t = h.tiles[b];
            const int64_t oz = t.z0 + z, oy = t.y0 + y, ox = t.x0 + x;
            if (oz < h.dz && oy < h.dy && ox < h.dx) {
                // (gz*gy)*gx*p in the reference's order (src/ml/infer.hpp:631-653)
                const float wzy = __fmul_rn(__ldg(h.gauss + z), __ldg(h.gauss + y));
                const float c = __fmul_rn(__fmul_rn(wzy, __ldg(h.gauss + x)), p);
                atomicAdd(h.acc + (oz * h.dy + oy) * h.dx + ox, c);
            }
        }
    }
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

int grid_for(int64_t n, int threads) {
    int64_t g = (n + threads - 1) / threads;
    if (g > 148 * 16) g = 148 * 16;
    if (g < 1) g = 1;
    return static_cast<int>(g);
}

}  // namespace

cudaError_t launch_tile_sums(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, const TileOrigin* tiles,
                             int ntiles, int P, unsigned long long* sums, cudaStream_t s) {
    const int64_t n = static_cast<int64_t>(P) * P * P;
    int gx = grid_for(n, kEwThreads * 8);
    count_launch();
    tile_sums_kernel<<<dim3(gx, ntiles), kEwThreads, 0, s>>>(vol, dz, dy, dx, tiles, P, sums);
    return cudaGetLastError();
}

cudaError_t launch_tile_norm(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, const TileOrigin* tiles,
                             int ntiles, int P, const unsigned long long* sums, uint8_t* l0, int64_t l0_batch_stride,
                             int l0_type, float* f32_out, cudaStream_t s) {
    const int64_t n = static_cast<int64_t>(P) * P * P;
    int gx = grid_for(n, kEwThreads * 4);
    count_launch();
    tile_norm_kernel<<<dim3(gx, ntiles), kEwThreads, 0, s>>>(vol, dz, dy, dx, tiles, P, sums, l0, l0_batch_stride,
                                                             l0_type, f32_out);
    return cudaGetLastError();
}

cudaError_t launch_in_finalize(const float* partials, int B, int nrec, int C, double count, const float* gamma,
                               const float* beta, float eps, float* ss, cudaStream_t s) {
    count_launch();
    in_finalize_kernel<<<dim3((C + 31) / 32, B), 1024, 0, s>>>(partials, nrec, C, count, gamma, beta, eps, ss);
    return cudaGetLastError();
}

cudaError_t launch_norm_act(const uint8_t* pre, int64_t pbs, int64_t pgs, GridGeom g, int C, int B, const float* ss,
                            float slope, NormDest d0, NormDest d1, unsigned* amax, cudaStream_t s) {
    const bool any_fp8 = (d0.ptr && d0.dtype == kOpE4M3) || (d1.ptr && d1.dtype == kOpE4M3);
    const int cpt = (any_fp8 || C % 16 == 0) ? 16 : 8;
    const int64_t total = static_cast<int64_t>(g.D) * g.H * g.W * (C / cpt) * B;
    count_launch();
    norm_act_kernel<<<grid_for(total, kEwThreads), kEwThreads, 0, s>>>(pre, pbs, pgs, g, C, B, ss, slope, d0, d1,
                                                                       amax, cpt);
    return cudaGetLastError();
}

cudaError_t launch_head_blend(const HeadParams& h, cudaStream_t s) {
    if (h.ncls < 1 || h.ncls > 2 || h.C > 64 || h.C % 8) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemcpyToSymbolAsync(c_head_w, h.wh, sizeof(float) * h.ncls * h.C, 0,
                                            cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return e;
    e = cudaMemcpyToSymbolAsync(c_head_b, h.bh, sizeof(float) * h.ncls, 0, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return e;
    const int64_t n = static_cast<int64_t>(h.P) * h.P * h.P * h.B;
    count_launch();
    head_blend_kernel<<<grid_for(n, kEwThreads), kEwThreads, 0, s>>>(h);
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

cudaError_t launch_accum_add(float* dst, const float* src, int64_t n, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    if ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) return cudaErrorMisalignedAddress;
    count_launch();
    accum_add_kernel<<<grid_for(n / 4 + 1, kEwThreads), kEwThreads, 0, s>>>(dst, src, n);
    return cudaGetLastError();
}

}  // namespace fxk
