// pack.cu — f32 NCDHW <-> padded group-plane conversions (see pack.cuh).
#include "pack.cuh"
#include "counters.hpp"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace fxk {

namespace {

int grid_for(int64_t n, int threads) {
    int64_t g = (n + threads - 1) / threads;
    if (g > 148 * 16) g = 148 * 16;
    if (g < 1) g = 1;
    return static_cast<int>(g);
}

__global__ void pack_kernel(const float* __restrict__ x, int B, int C, int D, int H, int W, uint8_t* out,
                            int64_t bs, int64_t gs, int dtype, float qs, int phase, int pHp, int pWp, int64_t ps) {
    const bool fp8 = dtype == kOpE4M3;
    const int cg = fp8 ? 16 : 8;
    const int G = (C + cg - 1) / cg;
    const int64_t vox = static_cast<int64_t>(D) * H * W;
    const int64_t total = vox * G * B;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t v = i % vox;
        const int64_t t = i / vox;
        const int g = static_cast<int>(t % G);
        const int b = static_cast<int>(t / G);
        const int xx = static_cast<int>(v % W);
        const int yy = static_cast<int>((v / W) % H);
        const int zz = static_cast<int>(v / (static_cast<int64_t>(W) * H));
        float f[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int c = g * cg + j;
            f[j] = (j < cg && c < C) ? x[(static_cast<int64_t>(b) * C + c) * vox + v] : 0.f;
        }
        const int zp = zz + 1, yp = yy + 1, xp = xx + 1;
        int64_t off;
        if (phase) {
            off = phase_cell_offset(phase, zp, yp, xp, pHp, pWp, ps);
        } else {
            off = ((static_cast<int64_t>(zp) * (H + 2) + yp) * (W + 2) + xp) * 16;
        }
        uint4 w;
        if (fp8) {
            w.x = pack_e4m3x4(f[0] * qs, f[1] * qs, f[2] * qs, f[3] * qs);
            w.y = pack_e4m3x4(f[4] * qs, f[5] * qs, f[6] * qs, f[7] * qs);
            w.z = pack_e4m3x4(f[8] * qs, f[9] * qs, f[10] * qs, f[11] * qs);
            w.w = pack_e4m3x4(f[12] * qs, f[13] * qs, f[14] * qs, f[15] * qs);
        } else {
            w = pack_cell16(f, dtype);
        }
        *reinterpret_cast<uint4*>(out + b * bs + g * gs + off) = w;
    }
}

__global__ void pack_first_kernel(const float* __restrict__ x, int B, int D, int H, int W, uint8_t* out, int64_t bs,
                                  int64_t gs, int dtype) {
    const int64_t vox = static_cast<int64_t>(D) * H * W;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < vox * B;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int b = static_cast<int>(i / vox);
        const int64_t v = i % vox;
        const int xx = static_cast<int>(v % W);
        const int yy = static_cast<int>((v / W) % H);
        const int zz = static_cast<int>(v / (static_cast<int64_t>(W) * H));
        const float* row = x + static_cast<int64_t>(b) * vox + (static_cast<int64_t>(zz) * H + yy) * W;
        const float taps[3] = {xx > 0 ? row[xx - 1] : 0.f, row[xx], xx + 1 < W ? row[xx + 1] : 0.f};
        uint4 c0, c1;
        first_layer_cells(taps, dtype, c0, c1);
        const int64_t r = ((static_cast<int64_t>(zz + 1) * (H + 2) + (yy + 1)) * (W + 2) + (xx + 1));
        *reinterpret_cast<uint4*>(out + b * bs + r * 16) = c0;
        *reinterpret_cast<uint4*>(out + b * bs + gs + r * 16) = c1;
    }
}

__global__ void unpack_kernel(const uint8_t* __restrict__ in, int64_t bs, int64_t gs, int dtype, float scale, int B,
                              int C, int D, int H, int W, float* __restrict__ y) {
    const bool fp8 = dtype == kOpE4M3;
    const int cg = fp8 ? 16 : 8;
    const int64_t vox = static_cast<int64_t>(D) * H * W;
    const int64_t total = vox * C * B;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t v = i % vox;
        const int64_t t = i / vox;
        const int c = static_cast<int>(t % C);
        const int b = static_cast<int>(t / C);
        const int xx = static_cast<int>(v % W);
        const int yy = static_cast<int>((v / W) % H);
        const int zz = static_cast<int>(v / (static_cast<int64_t>(W) * H));
        const int64_t r = ((static_cast<int64_t>(zz + 1) * (H + 2) + (yy + 1)) * (W + 2) + (xx + 1));
        const uint8_t* cell = in + b * bs + (c / cg) * gs + r * 16;
        float val;
        if (fp8) {
            __nv_fp8_e4m3 q;
            q.__x = cell[c % cg];
            val = static_cast<float>(q) * scale;
        } else if (dtype == kOpF16) {
            val = __half2float(reinterpret_cast<const __half*>(cell)[c % cg]);
        } else {
            val = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(cell)[c % cg]);
        }
        y[i] = val;
    }
}

__global__ void absmax_kernel(const float* __restrict__ x, int64_t n, unsigned* amax) {
    float m = 0.f;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        m = fmaxf(m, fabsf(x[i]));
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(amax, __float_as_uint(m));
}

}  // namespace

cudaError_t launch_pack(const float* x, int B, int C, int D, int H, int W, uint8_t* out, int64_t bs, int64_t gs,
                        int dtype, float qs, int phase, int pHp, int pWp, int64_t ps, cudaStream_t s) {
    const int cg = dtype == kOpE4M3 ? 16 : 8;
    const int64_t total = static_cast<int64_t>(D) * H * W * ((C + cg - 1) / cg) * B;
    count_launch();
    pack_kernel<<<grid_for(total, 256), 256, 0, s>>>(x, B, C, D, H, W, out, bs, gs, dtype, qs, phase, pHp, pWp, ps);
    return cudaGetLastError();
}

cudaError_t launch_pack_first(const float* x, int B, int D, int H, int W, uint8_t* out, int64_t bs, int64_t gs,
                              int dtype, cudaStream_t s) {
    const int64_t total = static_cast<int64_t>(D) * H * W * B;
    count_launch();
    pack_first_kernel<<<grid_for(total, 256), 256, 0, s>>>(x, B, D, H, W, out, bs, gs, dtype);
    return cudaGetLastError();
}

cudaError_t launch_unpack(const uint8_t* in, int64_t bs, int64_t gs, int dtype, float scale, int B, int C, int D,
                          int H, int W, float* y, cudaStream_t s) {
    const int64_t total = static_cast<int64_t>(D) * H * W * C * B;
    count_launch();
    unpack_kernel<<<grid_for(total, 256), 256, 0, s>>>(in, bs, gs, dtype, scale, B, C, D, H, W, y);
    return cudaGetLastError();
}

cudaError_t launch_absmax(const float* x, int64_t n, unsigned* amax, cudaStream_t s) {
    count_launch();
    absmax_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, n, amax);
    return cudaGetLastError();
}

}  // namespace fxk
