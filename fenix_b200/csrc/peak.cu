// peak.cu — the dense tcgen05 tensor rate of this GPU, measured with our own kernel: every SM keeps
// one CTA whose elected thread issues back-to-back M = 128 MMAs (kind::f8f6f4 with e4m3 operands,
// or kind::f16 with bf16 / f16) on operand tiles resident in shared memory into a TMEM accumulator.
// No global memory is touched inside the loop, so the rate is the tensor pipe's. At N = 256 it is
// the denominator the convolutions' tensor roofline is quoted against; narrower N (the 32- to
// 96-column MMAs of the narrow conv layers) gives the ceiling of that MMA shape, where the A tile's
// shared-memory read is spread over fewer columns of math.
#include "fenix_b200.h"
#include "counters.hpp"
#include "ptx.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <string>
#include <vector>

namespace fxh {
fx_status abi_error(int code, const std::string& msg);
}

namespace fxk {
namespace {

constexpr int kPeakM = 128, kPeakN = 256;
constexpr int kABytes = kPeakM * 32, kBBytes = kPeakN * 32;  // one MMA's K: 32 bytes per row

__global__ void __launch_bounds__(128, 1) tc_peak_kernel(int optype, int n_cols, long long n_mma, uint32_t* status) {
    __shared__ __align__(1024) uint8_t a_tile[kABytes];
    __shared__ __align__(1024) uint8_t b_tile[kBBytes];
    __shared__ uint64_t done;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5;
    // operand bytes: finite values of the type (e4m3 bytes with exponent < 15, 16-bit with a
    // mid-range exponent), varied so the multipliers toggle as on real data
    for (int i = threadIdx.x; i < kABytes + kBBytes; i += blockDim.x) {
        uint32_t h = static_cast<uint32_t>(i) * 2654435761u + blockIdx.x * 40503u;
        h ^= h >> 13;
        uint8_t v;
        if (optype == kOpE4M3) v = static_cast<uint8_t>((h & 0x87u) | (((h >> 8) % 14u + 1u) << 3));
        else v = (i & 1) ? static_cast<uint8_t>(0x38u | (h & 0x83u)) : static_cast<uint8_t>(h);
        (i < kABytes ? a_tile[i] : b_tile[i - kABytes]) = v;
    }
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&done), 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&tmem_base), kPeakN);
        tmem_relinquish();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy stores -> the MMA's reads
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) {
        const uint32_t leader = elect_one() ? 1u : 0u;
        // K-major, no swizzle: 8-row core matrices of 16-byte rows, SBO = 128 B between them, the two
        // 16-byte K halves LBO = rows x 16 B apart
        const uint64_t hi = (static_cast<uint64_t>(128 >> 4) << 32) | (static_cast<uint64_t>(1) << 46);
        const uint64_t adesc = hi | (static_cast<uint64_t>((kPeakM * 16) >> 4) << 16) | (smem_u32(a_tile) >> 4);
        const uint64_t bdesc = hi | (static_cast<uint64_t>((n_cols * 16) >> 4) << 16) | (smem_u32(b_tile) >> 4);
        const uint32_t idesc = instr_desc(kPeakM, n_cols, optype);
        const uint32_t d = tmem_base;
        uint32_t acc = 0;
        if (optype == kOpE4M3) {
            for (long long i = 0; i < n_mma; ++i) {
                mma_f8_if(leader, d, adesc, bdesc, idesc, acc);
                acc = 1;
            }
        } else {
            for (long long i = 0; i < n_mma; ++i) {
                mma_f16_if(leader, d, adesc, bdesc, idesc, acc);
                acc = 1;
            }
        }
        mma_commit_if(leader, smem_u32(&done));
        __syncwarp();
        // every MMA issued must have finished before TMEM is released; bounded wait
        const uint64_t t0 = globaltimer_ns();
        bool ok = false;
        while (!(ok = mbar_try_wait(smem_u32(&done), 0u)) && globaltimer_ns() - t0 < 20000000000ull) {
        }
        if (!ok && leader) set_status(status, kStatusTimeoutDrain);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kPeakN);
    }
}

}  // namespace
}  // namespace fxk

extern "C" fx_status fx_tc_rate(int device, int precision, int n_cols, double ms_per_run, int runs, double* best_tflops,
                                double* mean_tflops) {
    if (!best_tflops || runs < 1 || !(ms_per_run > 0.0) || n_cols < 16 || n_cols > fxk::kPeakN || n_cols % 16 ||
        (precision != FX_PREC_FP8 && precision != FX_PREC_BF16 && precision != FX_PREC_F16))
        return fxh::abi_error(FX_INVALID_ARGUMENT, "fx_tc_rate: bad argument");
    if (cudaSetDevice(device) != cudaSuccess) return fxh::abi_error(FX_INVALID_ARGUMENT, "fx_tc_peak: no such device");
    int major = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (major != 10) return fxh::abi_error(FX_UNSUPPORTED, "fx_tc_rate: needs an sm_100 GPU");
    const int optype = precision;  // fx_precision values are the kernel's operand types
    const double flop_per_mma = 2.0 * fxk::kPeakM * n_cols * (optype == fxk::kOpE4M3 ? 32 : 16);
    uint32_t* d_status = nullptr;
    cudaEvent_t e0, e1;
    if (cudaMalloc(&d_status, 4) != cudaSuccess) return fxh::abi_error(FX_INTERNAL, "fx_tc_rate: cudaMalloc");
    cudaMemset(d_status, 0, 4);
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    auto run = [&](long long n) -> double {  // ms of one launch of n MMAs per SM
        cudaEventRecord(e0);
        fxk::count_launch();
        fxk::tc_peak_kernel<<<sms, 128>>>(optype, n_cols, n, d_status);
        cudaEventRecord(e1);
        cudaEventSynchronize(e1);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        return ms;
    };
    // size the launch to ms_per_run from a short calibration launch
    const long long n0 = 1 << 16;
    run(n0);
    const double ms0 = std::max(run(n0), 1e-3);
    const long long n = std::max<long long>(n0, static_cast<long long>(static_cast<double>(n0) * ms_per_run / ms0));
    double best = 0.0, sum = 0.0;
    for (int r = 0; r < runs; ++r) {
        const double ms = run(n);
        const double tf = flop_per_mma * static_cast<double>(n) * sms / (ms * 1e-3) / 1e12;
        best = std::max(best, tf);
        sum += tf;
    }
    uint32_t status = 0;
    cudaMemcpy(&status, d_status, 4, cudaMemcpyDeviceToHost);
    const cudaError_t err = cudaGetLastError();
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(d_status);
    if (err != cudaSuccess) return fxh::abi_error(FX_INTERNAL, std::string("fx_tc_rate: ") + cudaGetErrorString(err));
    if (status) return fxh::abi_error(FX_INTERNAL, "fx_tc_rate: the final wait timed out");
    *best_tflops = best;
    if (mean_tflops) *mean_tflops = sum / runs;
    return FX_OK;
}

extern "C" fx_status fx_tc_peak(int device, int precision, double ms_per_run, int runs, double* best_tflops,
                                double* mean_tflops) {
    return fx_tc_rate(device, precision, fxk::kPeakN, ms_per_run, runs, best_tflops, mean_tflops);
}
