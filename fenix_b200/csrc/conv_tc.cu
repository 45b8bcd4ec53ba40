// conv_tc.cu — persistent warp-specialised tcgen05 implicit-GEMM kernel (see conv_tc.cuh for
// the data layout and the per-layer program it executes).
#include "conv_tc.cuh"
#include "ptx.cuh"

#include <cuda_runtime.h>

namespace fxk {

namespace {

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far above any legitimate stage wait

struct SmemCtl {
    uint64_t full[16];
    uint64_t empty[16];
    uint64_t accf[2];
    uint64_t acce[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ void unit_coords(const ConvParams& p, int unit, int& b, int& mu, int& nt) {
    nt = unit % p.n_tiles;
    const int t = unit / p.n_tiles;
    mu = t % p.n_units_m;
    b = t / p.n_units_m;
}

// Producer: one elected thread issues the bulk copies of every stage of every unit.
__device__ void producer_loop(const ConvParams& p, uint8_t* smem, SmemCtl* ctl, int n_units) {
    uint32_t k = 0;  // global stage counter
    const int Mtot = 128 * p.R;
    for (int unit = blockIdx.x; unit < n_units; unit += gridDim.x) {
        int b, mu, nt;
        unit_coords(p, unit, b, mu, nt);
        const int64_t q0 = p.row_begin + static_cast<int64_t>(mu) * Mtot;
        for (int s = 0; s < p.n_stages; ++s, ++k) {
            const int slot = k % p.n_pipe;
            const uint32_t ph = (k / p.n_pipe) & 1u;
            if (!mbar_wait(smem_u32(&ctl->empty[slot]), ph ^ 1u, &ctl->abort, kWaitLimitNs)) {
                set_status(p.status, kStatusTimeoutEmpty);
                ctl->abort = 1;
                goto drain;
            }
            const ConvStage st = p.stages[s];
            const ConvSrc& src = p.src[st.src];
            uint8_t* sbuf = smem + static_cast<size_t>(slot) * p.stage_bytes;
            const int64_t lo = q0 + st.row_off;
            const int64_t clo = lo < 0 ? 0 : lo;
            int64_t chi = lo + st.rows;
            if (chi > src.rows) chi = src.rows;
            const uint32_t a_bytes = chi > clo ? static_cast<uint32_t>((chi - clo) * 16) : 0u;
            const uint32_t total = a_bytes * static_cast<uint32_t>(st.ng) + static_cast<uint32_t>(st.b_bytes);
            const uint32_t fb = smem_u32(&ctl->full[slot]);
            mbar_arrive_expect_tx(fb, total);
            if (a_bytes) {
                const uint8_t* gbase = src.ptr + static_cast<int64_t>(b) * src.batch_stride + clo * 16;
                const uint32_t dbase = smem_u32(sbuf) + static_cast<uint32_t>((clo - lo) * 16);
                for (int g = 0; g < st.ng; ++g)
                    bulk_g2s(dbase + static_cast<uint32_t>(g * st.rows * 16),
                             gbase + static_cast<int64_t>(st.g0 + g) * src.group_stride, a_bytes, fb);
            }
            if (st.b_bytes)
                bulk_g2s(smem_u32(sbuf + p.stage_a_bytes), p.wpack + nt * p.wtile_bytes + st.b_off,
                         static_cast<uint32_t>(st.b_bytes), fb);
        }
    }
drain:
    // Drain: wait until every stage we filled has landed (the consumer may have aborted).
    const uint32_t n_issued = k;
    for (uint32_t j = (n_issued > static_cast<uint32_t>(p.n_pipe) ? n_issued - p.n_pipe : 0u); j < n_issued; ++j) {
        const int slot = j % p.n_pipe;
        if (!mbar_wait(smem_u32(&ctl->full[slot]), (j / p.n_pipe) & 1u, nullptr,
                       kWaitLimitNs)) {
            // An abort elsewhere is fine; a copy that never lands is recorded.
            if (!ctl->abort) set_status(p.status, kStatusTimeoutDrain);
            break;
        }
    }
}

// MMA issuer: one thread walks the program and issues tcgen05.mma into TMEM accumulators.
__device__ void mma_loop(const ConvParams& p, uint8_t* smem, SmemCtl* ctl, int n_units) {
    uint32_t k = 0;
    uint32_t j = 0;  // unit counter for accumulator slots
    const uint32_t tbase = ctl->tmem_base;
    const uint32_t slot_cols = static_cast<uint32_t>(p.R * p.N_tile);
    const uint32_t smem_base = smem_u32(smem);
    for (int unit = blockIdx.x; unit < n_units; unit += gridDim.x, ++j) {
        const int aslot = j % p.acc_slots;
        const uint32_t aph = (j / p.acc_slots) & 1u;
        if (!mbar_wait(smem_u32(&ctl->acce[aslot]), aph ^ 1u, &ctl->abort, kWaitLimitNs)) {
            set_status(p.status, kStatusTimeoutAccFree);
            ctl->abort = 1;
            break;
        }
        tc_fence_after();
        const uint32_t dcol0 = tbase + aslot * slot_cols;
        bool first = true;
        for (int s = 0; s < p.n_stages; ++s, ++k) {
            const int slot = k % p.n_pipe;
            if (!mbar_wait(smem_u32(&ctl->full[slot]), (k / p.n_pipe) & 1u, &ctl->abort, kWaitLimitNs)) {
                set_status(p.status, kStatusTimeoutFull);
                ctl->abort = 1;
                goto done;
            }
            tc_fence_after();
            {
                const ConvStage st = p.stages[s];
                const uint32_t sa = smem_base + static_cast<uint32_t>(slot * p.stage_bytes);
                const uint32_t sb = sa + static_cast<uint32_t>(p.stage_a_bytes);
                const uint32_t b_lbo = static_cast<uint32_t>(p.N_tile * 16);
                for (int m = 0; m < st.mma_count; ++m) {
                    const ConvMma mm = p.mmas[st.mma_begin + m];
                    for (int r = 0; r < p.R; ++r) {
                        const uint64_t adesc = smem_desc(sa + mm.a_off + r * 2048, mm.lbo, 128);
                        for (int n0 = 0; n0 < p.N_tile; n0 += 256) {
                            const int nn = p.N_tile - n0 < 256 ? p.N_tile - n0 : 256;
                            const uint64_t bdesc = smem_desc(sb + mm.b_off + n0 * 16, b_lbo, 128);
                            const uint32_t idesc = instr_desc(128, nn, p.optype);
                            const uint32_t d = dcol0 + r * p.N_tile + n0;
                            if (p.optype == kOpE4M3)
                                mma_f8(d, adesc, bdesc, idesc, first ? 0u : 1u);
                            else
                                mma_f16(d, adesc, bdesc, idesc, first ? 0u : 1u);
                        }
                    }
                    first = false;
                }
            }
            mma_commit(smem_u32(&ctl->empty[slot]));  // stage buffer free once these MMAs finish
        }
        mma_commit(smem_u32(&ctl->accf[aslot]));  // accumulator ready for the epilogue
    }
done:
    // Make sure nothing we issued is still running before TMEM is released.
    mma_commit(smem_u32(&ctl->drain));
    if (!mbar_wait(smem_u32(&ctl->drain), 0u, nullptr, kWaitLimitNs)) {
        // abort set by another role: still give in-flight MMAs time to finish
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(smem_u32(&ctl->drain), 0u) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
    }
}

// Butterfly "transpose-reduce" over 16 channels: on entry each lane holds 16 per-channel values
// of its row; on exit lane l holds the sum over all 32 rows of channel (l & 15).
__device__ __forceinline__ float warp_transpose_reduce16(float (&v)[16], int lane) {
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < off; ++i) {
            const float send = upper ? v[i] : v[i + off];
            const float keep = upper ? v[i + off] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 16);
}

__device__ __forceinline__ bool row_interior(int64_t row, int P2, int Wp, int Dp, int Hp) {
    const int64_t z = row / P2;
    const int rem = static_cast<int>(row - z * P2);
    const int y = rem / Wp;
    const int x = rem - y * Wp;
    return z >= 1 && z <= Dp - 2 && y >= 1 && y <= Hp - 2 && x >= 1 && x <= Wp - 2;
}

constexpr int kMaxChunks = 20;  // 320 columns / 16

__device__ void epilogue_loop(const ConvParams& p, SmemCtl* ctl, int n_units) {
    const int lane = threadIdx.x & 31;
    const int wq = (threadIdx.x >> 5) & 3;  // TMEM lane quarter this warp may access
    const uint32_t tbase = ctl->tmem_base;
    const uint32_t slot_cols = static_cast<uint32_t>(p.R * p.N_tile);
    const int Mtot = 128 * p.R;
    const int P2 = p.Hp * p.Wp;
    const int nch = p.N_tile / 16;
    uint32_t j = 0;
    for (int unit = blockIdx.x; unit < n_units; unit += gridDim.x, ++j) {
        int b, mu, nt;
        unit_coords(p, unit, b, mu, nt);
        const int aslot = j % p.acc_slots;
        if (!mbar_wait(smem_u32(&ctl->accf[aslot]), (j / p.acc_slots) & 1u, &ctl->abort, kWaitLimitNs)) {
            set_status(p.status, kStatusTimeoutAcc);
            ctl->abort = 1;
            return;
        }
        tc_fence_after();
        const int64_t q0 = p.row_begin + static_cast<int64_t>(mu) * Mtot;
        float s1[kMaxChunks], s2[kMaxChunks];
#pragma unroll
        for (int c = 0; c < kMaxChunks; ++c) s1[c] = s2[c] = 0.f;
        for (int r = 0; r < p.R; ++r) {
            const int64_t row = q0 + r * 128 + wq * 32 + lane;
            const bool valid = row < p.row_end && row_interior(row, P2, p.Wp, p.Dp, p.Hp);
            const uint32_t taddr = tbase + (static_cast<uint32_t>(wq * 32) << 16) + aslot * slot_cols + r * p.N_tile;
            int64_t zi = 0;
            int yi = 0, xi = 0;
            if (p.mode == kModeUpsample) {
                zi = row / P2;
                const int rem = static_cast<int>(row - zi * P2);
                yi = rem / p.Wp;
                xi = rem - yi * p.Wp;
            }
#pragma unroll 1
            for (int cc = 0; cc < nch; ++cc) {
                float v[16];
                tmem_ld16(taddr + cc * 16, v);
                const int n0 = nt * p.N_tile + cc * 16;  // global column of v[0]
                if (p.mode == kModePrenorm) {
                    if (p.col_scale) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) v[i] *= __ldg(p.col_scale + n0 + i);
                    }
                    if (valid) {
                        uint8_t* o = p.out + static_cast<int64_t>(b) * p.out_batch_stride + row * 16 +
                                     static_cast<int64_t>(n0 / 8) * p.out_group_stride;
#pragma unroll
                        for (int g = 0; g < 2; ++g)
                            *reinterpret_cast<uint4*>(o + g * p.out_group_stride) = pack_cell16(v + g * 8, kOpF16);
                    }
                    float q[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        v[i] = valid ? v[i] : 0.f;
                        q[i] = v[i] * v[i];
                    }
                    const float a1 = warp_transpose_reduce16(v, lane);
                    const float a2 = warp_transpose_reduce16(q, lane);
#pragma unroll
                    for (int c = 0; c < kMaxChunks; ++c)
                        if (c == cc) {
                            s1[c] += a1;
                            s2[c] += a2;
                        }
                } else if (valid) {  // kModeUpsample: column n = phase * cout + channel
                    const int a = n0 / p.cout;
                    const int co0 = n0 - a * p.cout;  // 16 consecutive channels of one phase
                    float mx = 0.f;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        if (p.col_scale) v[i] *= __ldg(p.col_scale + co0 + i);
                        v[i] += __ldg(p.bias + co0 + i);
                        mx = fmaxf(mx, fabsf(v[i]));
                    }
                    if (p.amax) atomicMax(p.amax, __float_as_uint(mx));
                    const int az = a >> 2, ay = (a >> 1) & 1, ax = a & 1;
                    const int64_t orow =
                        ((2 * zi - 1 + az) * static_cast<int64_t>(p.oHp) + (2 * yi - 1 + ay)) * p.oWp + (2 * xi - 1 + ax);
                    uint8_t* o = p.out + static_cast<int64_t>(b) * p.out_batch_stride + orow * 16;
                    if (p.out_type == kOpE4M3) {
                        const float s = p.out_qscale;
                        uint4 w;
                        w.x = pack_e4m3x4(v[0] * s, v[1] * s, v[2] * s, v[3] * s);
                        w.y = pack_e4m3x4(v[4] * s, v[5] * s, v[6] * s, v[7] * s);
                        w.z = pack_e4m3x4(v[8] * s, v[9] * s, v[10] * s, v[11] * s);
                        w.w = pack_e4m3x4(v[12] * s, v[13] * s, v[14] * s, v[15] * s);
                        *reinterpret_cast<uint4*>(o + static_cast<int64_t>(co0 / 16) * p.out_group_stride) = w;
                    } else {
#pragma unroll
                        for (int g = 0; g < 2; ++g)
                            *reinterpret_cast<uint4*>(o + static_cast<int64_t>(co0 / 8 + g) * p.out_group_stride) =
                                pack_cell16(v + g * 8, p.out_type);
                    }
                }
            }
        }
        // accumulator drained: hand it back to the MMA issuer
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ctl->acce[aslot]));
        if (p.mode == kModePrenorm) {
            float* dst = p.stats + ((static_cast<int64_t>(b) * p.n_units_m + mu) * 4 + wq) * p.stats_C * 2;
            for (int cc = 0; cc < nch; ++cc) {
                float a1 = 0.f, a2 = 0.f;
#pragma unroll
                for (int c = 0; c < kMaxChunks; ++c)
                    if (c == cc) {
                        a1 = s1[c];
                        a2 = s2[c];
                    }
                if (lane < 16) {
                    const int ch = nt * p.N_tile + cc * 16 + lane;
                    dst[ch * 2 + 0] = a1;
                    dst[ch * 2 + 1] = a2;
                }
            }
        }
    }
}

}  // namespace

__global__ void __launch_bounds__(kConvThreads, 1) conv_tc_kernel(const __grid_constant__ ConvParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw;
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(smem + static_cast<size_t>(p.n_pipe) * p.stage_bytes);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_units = p.batch * p.n_units_m * p.n_tiles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.n_pipe; ++i) {
            mbar_init(smem_u32(&ctl->full[i]), 1);
            mbar_init(smem_u32(&ctl->empty[i]), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_u32(&ctl->accf[i]), 1);
            mbar_init(smem_u32(&ctl->acce[i]), 4);
        }
        mbar_init(smem_u32(&ctl->drain), 1);
        ctl->abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&ctl->tmem_base), p.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == 0) {
        if (lane == 0) producer_loop(p, smem, ctl, n_units);
    } else if (warp == 1) {
        if (lane == 0) mma_loop(p, smem, ctl, n_units);
        __syncwarp();
    } else {
        epilogue_loop(p, ctl, n_units);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(ctl->tmem_base, p.tmem_cols);
    }
}

cudaError_t launch_conv_tc(const ConvParams& p, int grid, size_t smem_bytes, cudaStream_t stream) {
    static bool configured = false;
    if (!configured) {
        cudaError_t e =
            cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    conv_tc_kernel<<<grid, kConvThreads, smem_bytes, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace fxk
