// conv_tc.cu — persistent warp-specialised tcgen05 implicit-GEMM kernel (see conv_tc.cuh for
// the data layout and the per-layer program it executes).
#include "conv_tc.cuh"

#include <atomic>
#include "counters.hpp"
#include "ptx.cuh"

#include <cuda_runtime.h>

namespace fxk {

namespace {

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far above any legitimate stage wait

__device__ __forceinline__ uint64_t wait_limit(const ConvParams& p) { return p.wait_ns ? p.wait_ns : kWaitLimitNs; }

// Optional cycle accounting per role (build with -DFX_CONV_TRACE; p.trace gets 16 counters):
// [0] producer waiting for free stages, [1] producer issuing, [2] MMA waiting for drained
// accumulators, [3] MMA waiting for full stages, [4] MMA issuing, [5] epilogue waiting for
// accumulators, [6] epilogue draining, [7] MMAs issued, [8] units, [9] epilogue waiting for
// TMEM loads (part of [6]).
#ifdef FX_CONV_TRACE
#define FX_T0() const long long fx_t0_ = clock64()
#define FX_TADD(p, i) \
    do { \
        if ((p).trace) atomicAdd((p).trace + (i), static_cast<unsigned long long>(clock64() - fx_t0_)); \
    } while (0)
#define FX_TCNT(p, i, n) \
    do { \
        if ((p).trace) atomicAdd((p).trace + (i), static_cast<unsigned long long>(n)); \
    } while (0)
#else
#define FX_T0() ((void)0)
#define FX_TADD(p, i) ((void)0)
#define FX_TCNT(p, i, n) ((void)0)
#endif
constexpr int kMaxCols = 512;  // per-channel scale / bias table entries

struct SmemCtl {
    uint64_t full[16];
    uint64_t empty[16];
    uint64_t accf[2];
    uint64_t acce[2];
    uint64_t drain;
    uint64_t xready[2][2];  // fold epilogue: row exchange of [half][parity] published by its 4 warps
    uint64_t bres;          // z-plane fold: the resident weights have landed
    uint64_t never;         // failure self-test: a barrier nothing arrives at
    uint32_t tmem_base;
    int abort;
    alignas(16) float colscale[kMaxCols];
    alignas(16) float bias[kMaxCols];
};

// The barrier the MMA warp waits on for stage k: its full barrier, except in the failure self-test,
// where the first stage's wait goes to a barrier nothing arrives at.
__device__ __forceinline__ uint32_t stage_full_bar(const ConvParams& p, SmemCtl* ctl, int slot, uint32_t k) {
    return (p.stall_first_wait && k == 0) ? smem_u32(&ctl->never) : smem_u32(&ctl->full[slot]);
}

__device__ __forceinline__ void unit_coords(const ConvParams& p, int unit, int& b, int& mu, int& nt) {
    nt = unit % p.n_tiles;
    const int t = unit / p.n_tiles;
    mu = t % p.n_units_m;
    b = t / p.n_units_m;
}

// First output row of M unit mu. z-plane fold: unit = (group of R planes, 128-row segment of the
// plane's interior rows), its block r at + r * plane; otherwise R consecutive blocks of rows.
__device__ __forceinline__ int64_t unit_q0(const ConvParams& p, int mu) {
    if (p.zfold) {
        const int64_t P2 = static_cast<int64_t>(p.Hp) * p.Wp;
        const int zg = mu / p.zseg, seg = mu - zg * p.zseg;
        const int S = p.R / p.zplanes;
        return (1 + static_cast<int64_t>(zg) * p.zplanes) * P2 + (p.Wp + 1) + static_cast<int64_t>(seg) * 128 * S;
    }
    return p.row_begin + static_cast<int64_t>(mu) * p.block_rows * p.R;
}

// Producer warp: the whole warp walks the program (warp-uniform control flow); one elected lane
// issues the bulk copies of every stage of every unit.
__device__ void producer_loop(const ConvParams& p, uint8_t* smem, SmemCtl* ctl, int n_units) {
    const bool leader = elect_one();
    uint32_t k = 0;  // global stage counter
    if (p.zfold) {  // the weights of every tap, once per CTA
        if (leader) {
            mbar_arrive_expect_tx(smem_u32(&ctl->bres), static_cast<uint32_t>(p.bres_bytes));
            bulk_g2s(smem_u32(smem + p.bres_off), p.wpack, static_cast<uint32_t>(p.bres_bytes), smem_u32(&ctl->bres));
        }
        __syncwarp();
        const bool ok = mbar_wait(smem_u32(&ctl->bres), 0u, nullptr, wait_limit(p));
        if (!__all_sync(0xffffffffu, ok)) {
            if (leader) {
                set_status(p.status, kStatusTimeoutDrain);
                ctl->abort = 1;
            }
            return;
        }
    }
    for (int unit = blockIdx.x; unit < n_units; unit += gridDim.x) {
        int b, mu, nt;
        unit_coords(p, unit, b, mu, nt);
        const int64_t q0 = unit_q0(p, mu);
        for (int s = 0; s < p.n_stages; ++s, ++k) {
            const int slot = k % p.n_pipe;
            const uint32_t ph = (k / p.n_pipe) & 1u;
            {
                FX_T0();
                const bool ok = mbar_wait(smem_u32(&ctl->empty[slot]), ph ^ 1u, &ctl->abort, wait_limit(p));
                if (!__all_sync(0xffffffffu, ok)) {
                    if (leader) {
                        set_status(p.status, kStatusTimeoutEmpty);
                        ctl->abort = 1;
                    }
                    goto drain;
                }
                if (leader) FX_TADD(p, 0);
            }
            FX_T0();
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
            if (leader) {
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
                FX_TADD(p, 1);
            }
            __syncwarp();
        }
    }
drain:
    // Wait until every stage we filled has landed (the consumer may have aborted).
    const uint32_t n_issued = k;
    for (uint32_t j = (n_issued > static_cast<uint32_t>(p.n_pipe) ? n_issued - p.n_pipe : 0u); j < n_issued; ++j) {
        const int slot = j % p.n_pipe;
        const bool ok = mbar_wait(smem_u32(&ctl->full[slot]), (j / p.n_pipe) & 1u, nullptr, wait_limit(p));
        if (!__all_sync(0xffffffffu, ok)) {
            if (leader && !ctl->abort) set_status(p.status, kStatusTimeoutDrain);
            break;
        }
    }
}

// MMA warp: the whole warp runs this loop in lockstep so that its control flow and every operand
// are warp-uniform (program entries come from the parameter space, hence uniform registers); the
// MMA / commit instructions are predicated on the elected lane. R (M blocks per unit), the
// operand kind and the N split are compile-time, so issuing an MMA is a couple of uniform adds.
// FOLD: every program MMA is three MMAs of N = N_tile / 3 sharing the A tile (x-tap fold).
template <int R, bool F8, bool SPLIT, bool FOLD>
__device__ void mma_loop(const ConvParams& p, uint8_t* smem, SmemCtl* ctl, int n_units) {
    const uint32_t leader = elect_one() ? 1u : 0u;
    uint32_t k = 0;
    uint32_t j = 0;  // unit counter for accumulator slots
    const uint32_t tbase = ctl->tmem_base;
    const uint32_t slot_cols = static_cast<uint32_t>(R * p.N_tile);
    const uint32_t smem_base = smem_u32(smem);
    // descriptor high words: SBO = 128 B, version 1, no swizzle
    const uint64_t hi = (static_cast<uint64_t>(128 >> 4) << 32) | (static_cast<uint64_t>(1) << 46);
    const uint64_t b_lbo = static_cast<uint64_t>((p.N_tile * 16) >> 4) << 16;
    const uint32_t nf = static_cast<uint32_t>(p.N_tile / 3);  // FOLD: columns of each accumulator
    const uint32_t idesc0 = instr_desc(128, SPLIT ? 256 : (FOLD ? static_cast<int>(nf) : p.N_tile), p.optype);
    const uint32_t idesc1 = instr_desc(128, SPLIT ? p.N_tile - 256 : 16, p.optype);
    const uint32_t ncol = static_cast<uint32_t>(p.N_tile);
    const uint32_t brow16 = static_cast<uint32_t>(p.block_rows);  // M block stride in 16-byte rows
    const uint64_t bk1 = static_cast<uint64_t>((nf * 16) >> 4), bk2 = 2 * bk1;  // FOLD: B of x taps 1, 2
    for (int unit = blockIdx.x; unit < n_units; unit += gridDim.x, ++j) {
        const int aslot = j % p.acc_slots;
        const uint32_t aph = (j / p.acc_slots) & 1u;
        {
            FX_T0();
            const bool ok = mbar_wait(smem_u32(&ctl->acce[aslot]), aph ^ 1u, &ctl->abort, wait_limit(p));
            if (!__all_sync(0xffffffffu, ok)) {
                if (leader) {
                    set_status(p.status, kStatusTimeoutAccFree);
                    ctl->abort = 1;
                }
                break;
            }
            if (leader) FX_TADD(p, 2);
        }
        tc_fence_after();
        const uint32_t dcol0 = tbase + aslot * slot_cols;
        uint32_t acc = 0;
        bool aborted = false;
        for (int s = 0; s < p.n_stages; ++s, ++k) {
            const int slot = k % p.n_pipe;
            const int mb = p.stages[s].mma_begin, mc = p.stages[s].mma_count;
            {
                FX_T0();
                const bool ok =
                    mbar_wait(stage_full_bar(p, ctl, slot, k), (k / p.n_pipe) & 1u, &ctl->abort, wait_limit(p));
                if (!__all_sync(0xffffffffu, ok)) {
                    if (leader) {
                        set_status(p.status, kStatusTimeoutFull);
                        ctl->abort = 1;
                    }
                    aborted = true;
                    break;
                }
                if (leader) FX_TADD(p, 3);
            }
            tc_fence_after();
            FX_T0();
            const uint32_t sa16 = (smem_base + static_cast<uint32_t>(slot * p.stage_bytes)) >> 4;
            const uint32_t sb16 = sa16 + (static_cast<uint32_t>(p.stage_a_bytes) >> 4);
            const uint64_t ahi = hi + sa16;          // + packed (lbo, A offset) per MMA
            const uint64_t bhi = hi | b_lbo;         // + (stage B base + B offset) per MMA
            for (int m = mb; m < mb + mc; ++m) {
                const ConvMma mm = p.mmas[m];
                const uint64_t adesc = ahi + mm.a;  // lbo lands in bits 16..29, the address in 0..13
                const uint64_t bdesc = bhi + (sb16 + mm.b);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const uint64_t ad = adesc + static_cast<uint64_t>(r * brow16);
                    const uint32_t d = dcol0 + static_cast<uint32_t>(r) * ncol;
                    if (FOLD) {
                        if (F8) mma3_f8_if(leader, d, d + nf, d + 2 * nf, ad, bdesc, bdesc + bk1, bdesc + bk2, idesc0, acc);
                        else mma3_f16_if(leader, d, d + nf, d + 2 * nf, ad, bdesc, bdesc + bk1, bdesc + bk2, idesc0, acc);
                        continue;
                    }
                    if (F8) mma_f8_if(leader, d, ad, bdesc, idesc0, acc);
                    else mma_f16_if(leader, d, ad, bdesc, idesc0, acc);
                    if (SPLIT) {
                        const uint64_t bd1 = bdesc + static_cast<uint64_t>((256 * 16) >> 4);
                        if (F8) mma_f8_if(leader, d + 256, ad, bd1, idesc1, acc);
                        else mma_f16_if(leader, d + 256, ad, bd1, idesc1, acc);
                    }
                }
                acc = 1;
            }
            mma_commit_if(leader, smem_u32(&ctl->empty[slot]));  // stage buffer free once these MMAs finish
            if (leader) {
                FX_TADD(p, 4);
                FX_TCNT(p, 7, mc * R * (FOLD ? 3 : 1));
            }
        }
        if (aborted) break;
        mma_commit_if(leader, smem_u32(&ctl->accf[aslot]));  // accumulator ready for the epilogue
    }
    // Make sure nothing we issued is still running before TMEM is released.
    mma_commit_if(leader, smem_u32(&ctl->drain));
    if (leader) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(smem_u32(&ctl->drain), 0u) && globaltimer_ns() - t0 < wait_limit(p)) {
        }
    }
    __syncwarp();
}

// MMA warp of the z-plane fold: stage j of a unit holds input plane j - 1 relative to the unit's
// first block plane; each program entry (ky, kx, group pair) and segment is one A tile that feeds
// block (segment, j - kz) with tap kz for every kz in [kz_lo, kz_hi] = [max(0, j - Z + 1), min(2, j)].
// Those taps are ONE MMA of N = (kz_hi - kz_lo + 1) N_tile: the resident weights hold the three kz
// taps of an entry as consecutive rows of B, and the blocks of a segment sit at descending TMEM
// columns (plane p at (Z - 1 - p) N_tile), so accumulator columns [kz N_tile, (kz + 1) N_tile) of
// the MMA are plane j - kz's. The first entry of a stage with kz_lo = 0 is split in two: plane j
// starts its accumulator with tap 0 alone while the planes below keep accumulating. The segments
// alternate, so consecutive MMAs hit different accumulators. The issue stream is the bound of this
// loop, so the stages are unrolled (Z and S compile-time: each stage's tap range is a constant) and
// one elected thread issues while the warp waits.
template <bool F8, int Z>
__device__ void mma_loop_z(const ConvParams& p, uint8_t* smem, SmemCtl* ctl, int n_units) {
    constexpr int S = 2;
    const bool leader = elect_one();
    uint32_t k = 0;
    uint32_t j = 0;
    const uint32_t tbase = ctl->tmem_base;
    const uint32_t ncol = static_cast<uint32_t>(p.N_tile);
    const uint32_t slot_cols = static_cast<uint32_t>(S * Z) * ncol;
    const uint32_t smem_base = smem_u32(smem);
    const uint64_t hi = (static_cast<uint64_t>(128 >> 4) << 32) | (static_cast<uint64_t>(1) << 46);
    // resident weights: per entry [K half][kz 0..2][N_tile rows][16 B]; taps kz_lo.. of one MMA are
    // consecutive rows of B, so the K-half stride (LBO) spans all three
    const uint64_t b_lbo = static_cast<uint64_t>((3 * p.zkstride) >> 4) << 16;
    const uint32_t idesc1 = instr_desc(128, p.N_tile, p.optype);
    const uint32_t idesc2 = instr_desc(128, 2 * p.N_tile, p.optype);
    const uint32_t idesc3 = instr_desc(128, 3 * p.N_tile, p.optype);
    const uint64_t bres = (hi | b_lbo) + ((smem_base + static_cast<uint32_t>(p.bres_off)) >> 4);
    const uint64_t kzs = static_cast<uint64_t>(p.zkstride >> 4);  // rows of tap kz -> kz + 1
    const int nent = p.n_mmas;
    {
        const bool ok = mbar_wait(smem_u32(&ctl->bres), 0u, &ctl->abort, wait_limit(p));
        if (!__all_sync(0xffffffffu, ok)) {
            if (leader) {
                set_status(p.status, kStatusTimeoutFull);
                ctl->abort = 1;
            }
            n_units = 0;  // issue nothing; fall through to the drain
        }
    }
    tc_fence_after();
    for (int unit = blockIdx.x; unit < n_units; unit += gridDim.x, ++j) {
        const int aslot = j % p.acc_slots;
        const uint32_t aph = (j / p.acc_slots) & 1u;
        {
            FX_T0();
            const bool ok = mbar_wait(smem_u32(&ctl->acce[aslot]), aph ^ 1u, &ctl->abort, wait_limit(p));
            if (!__all_sync(0xffffffffu, ok)) {
                if (leader) {
                    set_status(p.status, kStatusTimeoutAccFree);
                    ctl->abort = 1;
                }
                break;
            }
            if (leader) FX_TADD(p, 2);
        }
        tc_fence_after();
        const uint32_t dcol0 = tbase + aslot * slot_cols;
        bool aborted = false;
#pragma unroll
        for (int s = 0; s < Z + 2; ++s, ++k) {
            const int slot = k % p.n_pipe;
            {
                FX_T0();
                const bool ok =
                    mbar_wait(stage_full_bar(p, ctl, slot, k), (k / p.n_pipe) & 1u, &ctl->abort, wait_limit(p));
                if (!__all_sync(0xffffffffu, ok)) {
                    if (leader) {
                        set_status(p.status, kStatusTimeoutFull);
                        ctl->abort = 1;
                    }
                    aborted = true;
                    break;
                }
                if (leader) FX_TADD(p, 3);
            }
            tc_fence_after();
            FX_T0();
            const int kz_lo = s - (Z - 1) > 0 ? s - (Z - 1) : 0;  // constants once s is unrolled
            const int nz = (s < 2 ? s : 2) - kz_lo + 1;
            if (leader) {
                const uint64_t ahi = hi + ((smem_base + static_cast<uint32_t>(slot * p.stage_bytes)) >> 4);
                const uint64_t bbase = bres + static_cast<uint64_t>(kz_lo) * kzs;
                // plane s - kz_lo of segment 0; planes below it follow at + ncol, + 2 ncol
                const uint32_t dtop = dcol0 + static_cast<uint32_t>(Z - 1 - (s - kz_lo)) * ncol;
                const uint32_t idn = nz == 3 ? idesc3 : nz == 2 ? idesc2 : idesc1;
                int e0 = 0;
                if (kz_lo == 0) {
                    // first entry: plane s starts its accumulator with tap kz 0 alone; the planes
                    // below it (taps 1, 2) keep accumulating
                    const ConvMma mm = p.mmas[0];
#pragma unroll
                    for (int sg = 0; sg < S; ++sg) {
                        const uint64_t ad = ahi + mm.a + static_cast<uint64_t>(sg * 128);
                        const uint32_t d0 = dtop + static_cast<uint32_t>(sg * Z) * ncol;
                        if (F8) mma_f8_if(1u, d0, ad, bbase + mm.b, idesc1, 0u);
                        else mma_f16_if(1u, d0, ad, bbase + mm.b, idesc1, 0u);
                        if (nz > 1) {
                            if (F8) mma_f8_if(1u, d0 + ncol, ad, bbase + mm.b + kzs, nz == 3 ? idesc2 : idesc1, 1u);
                            else mma_f16_if(1u, d0 + ncol, ad, bbase + mm.b + kzs, nz == 3 ? idesc2 : idesc1, 1u);
                        }
                    }
                    e0 = 1;
                }
                for (int e = e0; e < nent; ++e) {
                    const ConvMma mm = p.mmas[e];
                    const uint64_t bb = bbase + mm.b;
                    const uint64_t a0 = ahi + mm.a;
#pragma unroll
                    for (int sg = 0; sg < S; ++sg) {
                        const uint64_t ad = a0 + static_cast<uint64_t>(sg * 128);
                        const uint32_t d0 = dtop + static_cast<uint32_t>(sg * Z) * ncol;
                        if (F8) mma_f8_if(1u, d0, ad, bb, idn, 1u);
                        else mma_f16_if(1u, d0, ad, bb, idn, 1u);
                    }
                }
            }
            __syncwarp();
            mma_commit_if(leader ? 1u : 0u, smem_u32(&ctl->empty[slot]));
            if (leader) {
                FX_TADD(p, 4);
                FX_TCNT(p, 7, (nent + (kz_lo == 0 && nz > 1 ? 1 : 0)) * S);
            }
        }
        if (aborted) break;
        mma_commit_if(leader ? 1u : 0u, smem_u32(&ctl->accf[aslot]));
    }
    mma_commit_if(leader ? 1u : 0u, smem_u32(&ctl->drain));
    if (leader) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(smem_u32(&ctl->drain), 0u) && globaltimer_ns() - t0 < wait_limit(p)) {
        }
    }
    __syncwarp();
}

// Butterfly "transpose-reduce" over 16 channels: on entry each lane holds 16 per-channel values
// of its row; on exit lane l holds the sum over all 32 lanes of channel (l & 15).
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

// (z, y, x) of a row of the padded row space by multiply-high division (exact for row * d < 2^64).
struct RowDecomp {
    uint64_t mP2, mWp;
    uint32_t P2, Wp;
    __device__ __forceinline__ void split_plane(uint32_t rem, uint32_t& y, uint32_t& x) const {
        y = static_cast<uint32_t>(__umul64hi(rem, mWp));
        x = rem - y * Wp;
    }
    __device__ __forceinline__ void split(uint32_t row, uint32_t& z, uint32_t& y, uint32_t& x) const {
        z = static_cast<uint32_t>(__umul64hi(row, mP2));
        const uint32_t rem = row - z * P2;
        y = static_cast<uint32_t>(__umul64hi(rem, mWp));
        x = rem - y * Wp;
    }
};

// Epilogue for N_tile = 16 * NCH columns: 8 warps drain the TMEM accumulator of each unit
// (warp w owns TMEM lanes 32 (w % 4) .. +31, i.e. one output row per thread per M block). The two
// warps of a lane quarter split the work: alternate M blocks when a unit has several (SPLITC
// false), alternate 16-column chunks when it has one (SPLITC true). Each warp writes one
// statistics record per unit; entries of channels it did not handle are written as zeros.
template <int NCH, bool SPLITC>
__device__ void epilogue_loop(const ConvParams& p, SmemCtl* ctl, int n_units) {
    const int lane = threadIdx.x & 31;
    const int wq = (threadIdx.x >> 5) & 3;            // TMEM lane quarter of this warp (warp id % 4)
    const int half = ((threadIdx.x >> 5) - 2) >> 2;   // which of the two warps of the quarter
    const uint32_t tbase = ctl->tmem_base;
    const uint32_t slot_cols = static_cast<uint32_t>(p.R * p.N_tile);
    const int64_t P2r = static_cast<int64_t>(p.Hp) * p.Wp;
    constexpr bool kFold = NCH <= 4;  // narrow tiles: the z-plane fold, several M blocks per unit
    const bool zfold = kFold && p.zfold;
    const int zpl = zfold ? p.zplanes : 1;
    const int lzp = zpl == 4 ? 2 : (zpl == 2 ? 1 : 0);  // log2(zplanes): 2 or 4 planes per fold unit
    RowDecomp rd;
    rd.P2 = static_cast<uint32_t>(p.Hp * p.Wp);
    rd.Wp = static_cast<uint32_t>(p.Wp);
    rd.mP2 = ~0ull / rd.P2 + 1;
    rd.mWp = ~0ull / rd.Wp + 1;
    const uint32_t zmax = static_cast<uint32_t>(p.Dp - 2), ymax = static_cast<uint32_t>(p.Hp - 2),
                   xmax = static_cast<uint32_t>(p.Wp - 2);
    const bool prenorm = p.mode == kModePrenorm;
    constexpr int kMy = SPLITC ? NCH / 2 : NCH;  // chunks of an M block handled by this warp
    constexpr int kCs = SPLITC ? 2 : 1;           // chunk stride
    const int c0 = SPLITC ? half : 0;             // first chunk
    const int rb = SPLITC ? 0 : half, rs = SPLITC ? 1 : 2;
    // rs * 128 rows as (lines, voxels) within a padded plane, for the per-block row advance
    uint32_t sty, stx;
    rd.split_plane(static_cast<uint32_t>(rs * 128) % rd.P2, sty, stx);
    constexpr bool kAccR = kMy <= 2;         // sum over M blocks in registers, one butterfly per unit
    constexpr int kGrp = kMy <= 4 ? kMy : (kMy % 4 == 0 ? 4 : 2);  // chunks loaded from TMEM per wait
    constexpr int kR = kAccR ? kMy : 1;
    const bool e4out = p.out_type == kOpE4M3;
    // prenorm: a per-column scale table, or one scale for all columns (the per-channel part then
    // travels to the InstanceNorm statistics, which a per-channel factor does not change)
    const bool percol = p.col_scale != nullptr;
    const float acc_scale = p.acc_scale;
    const int32_t oP2 = p.oHp * p.oWp;  // upsample: padded plane of the output grid
    // upsample: factor along each axis and the bit of a phase index that holds each axis's parity
    const int um = p.up_mask;
    const int uz = (um & 4) ? 2 : 1, uy = (um & 2) ? 2 : 1, ux = (um & 1) ? 2 : 1;
    const int bx = 0, by = (um & 1) ? 1 : 0, bz = by + ((um & 2) ? 1 : 0);
    // InstanceNorm partial sums accumulate over all units of one (batch item, N tile) run of this
    // CTA; a run ends in one flush: butterfly, then add into this warp's slot of the CTA's record
    // [b][blockIdx.x][stat_recs] (records start at zero; the statistics pass clears what it reads).
    // Four records per CTA when the warp pair splits the chunks (both warps of a lane quarter fill
    // one record, each its own channels), eight otherwise.
    float s1[kMy], s2[kMy];
    float r1[kR][16], r2[kR][16];
#pragma unroll
    for (int c = 0; c < kMy; ++c) s1[c] = s2[c] = 0.f;
#pragma unroll
    for (int c = 0; c < kR; ++c)
#pragma unroll
        for (int i = 0; i < 16; ++i) r1[c][i] = r2[c][i] = 0.f;
    int run_b = -1, run_nt = 0;
    auto flush = [&]() {
        if constexpr (kAccR) {
#pragma unroll
            for (int c = 0; c < kMy; ++c) {
                s1[c] = warp_transpose_reduce16(r1[c], lane);
                s2[c] = warp_transpose_reduce16(r2[c], lane);
            }
#pragma unroll
            for (int c = 0; c < kR; ++c)
#pragma unroll
                for (int i = 0; i < 16; ++i) r1[c][i] = r2[c][i] = 0.f;
        }
        const bool shared = SPLITC && p.stat_recs == kStatRecsPerUnit / 2;
        float* dst = p.stats + ((static_cast<int64_t>(run_b) * gridDim.x + blockIdx.x) * p.stat_recs +
                                (shared ? wq : half * 4 + wq)) *
                                   p.stats_C * 2;
        if (lane < 16) {
#pragma unroll
            for (int c = 0; c < kMy; ++c) {
                float2* q = reinterpret_cast<float2*>(dst + (run_nt * p.N_tile + (c0 + c * kCs) * 16 + lane) * 2);
                const float2 o = *q;
                *q = make_float2(o.x + s1[c], o.y + s2[c]);
            }
        }
#pragma unroll
        for (int c = 0; c < kMy; ++c) s1[c] = s2[c] = 0.f;
    };
    uint32_t j = 0;
    for (int unit = blockIdx.x; unit < n_units; unit += gridDim.x, ++j) {
        int b, mu, nt;
        unit_coords(p, unit, b, mu, nt);
        if (prenorm && (b != run_b || nt != run_nt)) {
            if (run_b >= 0) flush();
            run_b = b;
            run_nt = nt;
        }
        const int aslot = j % p.acc_slots;
        {
            FX_T0();
            if (!mbar_wait(smem_u32(&ctl->accf[aslot]), (j / p.acc_slots) & 1u, &ctl->abort, wait_limit(p))) {
                set_status(p.status, kStatusTimeoutAcc);
                ctl->abort = 1;
                return;
            }
            if (threadIdx.x == 64) FX_TADD(p, 5);
        }
        tc_fence_after();
        FX_T0();
        const int64_t q0 = unit_q0(p, mu);
        // z-plane fold: block r owns plane zb + r only (a segment longer than a small plane's
        // interior reaches into the next plane, whose rows its own block counts)
        const uint32_t zb = zfold ? 1u + static_cast<uint32_t>((mu / p.zseg) * p.zplanes) : 0u;
        // Every plane of a fold segment has the same in-plane offset o, so (y, x) and ownership
        // (o inside the plane) are decided once per segment; a block then only checks its plane.
        uint32_t zok = 0;  // bit sg: this thread's row of segment sg is an output
        if (zfold) {
            const uint32_t o0 = static_cast<uint32_t>(q0 - static_cast<int64_t>(zb) * P2r) + wq * 32 + lane;
#pragma unroll
            for (int sg = 0; sg < 2; ++sg) {
                const uint32_t o = o0 + sg * 128;
                uint32_t y, x;
                rd.split_plane(o, y, x);
                const bool ok = o < rd.P2 && y >= 1 && y <= ymax && x >= 1 && x <= xmax;
                zok |= (ok ? 1u : 0u) << sg;
            }
        }
        // Regular tiling of narrow tiles: the blocks are visited in order rb, rb + rs, ..., each
        // rs * 128 rows after the previous one, so this thread's (z, y, x) advances by a
        // mixed-radix add.
        // Rows start at row_begin (plane 1) and row < row_end caps the plane, so only (y, x) are kept.
        int64_t crow = 0;
        uint32_t cy = 0, cx = 0;
        if (kFold && !zfold) {
            crow = q0 + static_cast<int64_t>(rb) * 128 + wq * 32 + lane;
            uint32_t cz;
            rd.split(static_cast<uint32_t>(crow), cz, cy, cx);
        }
        // M block r (called once per block, in order): its row for this thread, whether that row is
        // an output of this block, and its TMEM column block (fold: segment r >> lzp, plane
        // r & (zplanes - 1), planes at descending columns)
        auto locate = [&](int r, int64_t& row, bool& valid, int& rc) {
            if (zfold) {
                const int sg = r >> lzp, rz = r & (zpl - 1);
                row = q0 + sg * 128 + rz * P2r + wq * 32 + lane;
                valid = ((zok >> sg) & 1u) && zb + static_cast<uint32_t>(rz) <= zmax;
                rc = r + zpl - 1 - 2 * rz;
            } else if constexpr (!kFold) {  // wide tiles (one or two blocks per unit): split directly
                row = q0 + static_cast<int64_t>(r) * 128 + wq * 32 + lane;
                uint32_t z, y, x;
                rd.split(static_cast<uint32_t>(row), z, y, x);
                valid = row < p.row_end && z >= 1 && z <= zmax && y >= 1 && y <= ymax && x >= 1 && x <= xmax;
                rc = r;
            } else {
                row = crow;
                valid = row >= p.row_begin && row < p.row_end && cy >= 1 && cy <= ymax && cx >= 1 && cx <= xmax;
                rc = r;
                crow += static_cast<int64_t>(rs) * 128;
                cx += stx;
                if (cx >= rd.Wp) {
                    cx -= rd.Wp;
                    ++cy;
                }
                cy += sty;
                if (cy >= static_cast<uint32_t>(p.Hp)) cy -= static_cast<uint32_t>(p.Hp);
            }
        };
        const int cbase = nt * p.N_tile;  // first global column of this tile
        // prenorm, one chunk per block: the TMEM reads of kBlk blocks share one wait
        constexpr int kBlk = 4;
        int r_first = rb;
        if constexpr (kMy == 1 && kAccR) {
            if (prenorm) {
                for (; r_first + (kBlk - 1) * rs < p.R; r_first += kBlk * rs) {
                    int64_t rowv[kBlk];
                    bool validv[kBlk];
                    uint32_t raw[kBlk][16];
#pragma unroll
                    for (int k = 0; k < kBlk; ++k) {
                        int rc;
                        locate(r_first + k * rs, rowv[k], validv[k], rc);
                        tmem_ld16_nowait(tbase + (static_cast<uint32_t>(wq * 32) << 16) + aslot * slot_cols +
                                             rc * p.N_tile + c0 * 16,
                                         raw[k]);
                    }
                    tmem_wait();
#pragma unroll
                    for (int k = 0; k < kBlk; ++k) tmem_regs_ready(raw[k]);
#pragma unroll
                    for (int k = 0; k < kBlk; ++k) {
                        // invalid rows (halo, other planes, past the end; their accumulators may hold
                        // sums over uninitialised memory, NaN included) are selected to zero
                        float v[16];
                        if (percol) {
#pragma unroll
                            for (int i = 0; i < 16; ++i)
                                v[i] = validv[k] ? __uint_as_float(raw[k][i]) * ctl->colscale[cbase + c0 * 16 + i] : 0.f;
                        } else {
#pragma unroll
                            for (int i = 0; i < 16; ++i) v[i] = validv[k] ? __uint_as_float(raw[k][i]) * acc_scale : 0.f;
                        }
                        if (validv[k]) {
                            uint8_t* o = p.out + static_cast<int64_t>(b) * p.out_batch_stride + rowv[k] * 16 +
                                         static_cast<int64_t>((cbase + c0 * 16) / 8) * p.out_group_stride;
                            *reinterpret_cast<uint4*>(o) = pack_cell_f16_sat(v);
                            *reinterpret_cast<uint4*>(o + p.out_group_stride) = pack_cell_f16_sat(v + 8);
                        }
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            r1[0][i] += v[i];
                            r2[0][i] = fmaf(v[i], v[i], r2[0][i]);
                        }
                    }
                }
            }
        }
        for (int r = r_first; r < p.R; r += rs) {
            int64_t row;
            bool valid;
            int rc;
            locate(r, row, valid, rc);
            const uint32_t taddr =
                tbase + (static_cast<uint32_t>(wq * 32) << 16) + aslot * slot_cols + rc * p.N_tile;
            // upsample: phase-0 output cell of this input voxel (u (z - 1) + 1 per axis in the padded grid)
            uint8_t* ob = nullptr;
            if (!prenorm && valid) {  // upsample runs no fold: the row splits directly
                uint32_t z, y, x;
                rd.split(static_cast<uint32_t>(row), z, y, x);
                ob = p.out + static_cast<int64_t>(b) * p.out_batch_stride +
                     ((static_cast<int64_t>(uz * (z - 1) + 1) * p.oHp + (uy * (y - 1) + 1)) * p.oWp +
                      (ux * (x - 1) + 1)) * 16;
            }
#pragma unroll
            for (int g0 = 0; g0 < kMy; g0 += kGrp) {
                uint32_t raw[kGrp][16];
#ifdef FX_CONV_TRACE
                const long long fx_tl0_ = clock64();
#endif
#pragma unroll
                for (int c = 0; c < kGrp; ++c) tmem_ld16_nowait(taddr + (c0 + (g0 + c) * kCs) * 16, raw[c]);
                tmem_wait();
#ifdef FX_CONV_TRACE
                if (threadIdx.x == 64 && p.trace)
                    atomicAdd(p.trace + 9, static_cast<unsigned long long>(clock64() - fx_tl0_));
#endif
#pragma unroll
                for (int c = 0; c < kGrp; ++c) tmem_regs_ready(raw[c]);
#pragma unroll
                for (int c = 0; c < kGrp; ++c) {
                    const int ci = g0 + c;              // position among this warp's chunks
                    const int cc = c0 + ci * kCs;       // chunk within the tile
                    float v[16];
                    if (prenorm) {
                        if (percol) {
#pragma unroll
                            for (int i = 0; i < 16; ++i)
                                v[i] = __uint_as_float(raw[c][i]) * ctl->colscale[cbase + cc * 16 + i];
                        } else {
#pragma unroll
                            for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(raw[c][i]) * acc_scale;
                        }
                        if (valid) {
                            uint8_t* o = p.out + static_cast<int64_t>(b) * p.out_batch_stride + row * 16 +
                                         static_cast<int64_t>((cbase + cc * 16) / 8) * p.out_group_stride;
                            *reinterpret_cast<uint4*>(o) = pack_cell_f16_sat(v);
                            *reinterpret_cast<uint4*>(o + p.out_group_stride) = pack_cell_f16_sat(v + 8);
                        }
                        if constexpr (kAccR) {
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const float t = valid ? v[i] : 0.f;
                                r1[ci][i] += t;
                                r2[ci][i] = fmaf(t, t, r2[ci][i]);
                            }
                        } else {
                            float q[16];
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                v[i] = valid ? v[i] : 0.f;
                                q[i] = v[i] * v[i];
                            }
                            s1[ci] += warp_transpose_reduce16(v, lane);
                            s2[ci] += warp_transpose_reduce16(q, lane);
                        }
                    } else if (valid) {  // kModeUpsample: column n = phase * cout + channel
                        const int n0 = cbase + cc * 16;
                        const int a = n0 / p.cout;
                        const int co0 = n0 - a * p.cout;  // 16 consecutive channels of one phase
                        // scale and bias already include the e4m3 output scale
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            v[i] = fmaf(__uint_as_float(raw[c][i]), ctl->colscale[co0 + i], ctl->bias[co0 + i]);
                        if (p.amax) {
                            float mx = 0.f;
#pragma unroll
                            for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(v[i]));
                            if (e4out) mx /= p.out_qscale;
                            atomicMax(p.amax, __float_as_uint(mx));
                        }
                        const int az = uz == 2 ? (a >> bz) & 1 : 0, ay = uy == 2 ? (a >> by) & 1 : 0,
                                  ax = ux == 2 ? (a >> bx) & 1 : 0;
                        uint8_t* o = ob + static_cast<int64_t>(az * oP2 + ay * p.oWp + ax) * 16;
                        if (e4out) {
                            uint4 w;
                            w.x = pack_e4m3x4(v[0], v[1], v[2], v[3]);
                            w.y = pack_e4m3x4(v[4], v[5], v[6], v[7]);
                            w.z = pack_e4m3x4(v[8], v[9], v[10], v[11]);
                            w.w = pack_e4m3x4(v[12], v[13], v[14], v[15]);
                            *reinterpret_cast<uint4*>(o + static_cast<int64_t>(co0 / 16) * p.out_group_stride) = w;
                        } else {
                            *reinterpret_cast<uint4*>(o + static_cast<int64_t>(co0 / 8) * p.out_group_stride) =
                                pack_cell16(v, p.out_type);
                            *reinterpret_cast<uint4*>(o + static_cast<int64_t>(co0 / 8 + 1) * p.out_group_stride) =
                                pack_cell16(v + 8, p.out_type);
                        }
                    }
                }
            }
        }
        // accumulator drained: hand it back to the MMA issuer
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ctl->acce[aslot]));
        if (threadIdx.x == 64) {
            FX_TADD(p, 6);
            FX_TCNT(p, 8, 1);
        }
    }
    if (prenorm && run_b >= 0) flush();
}

// Epilogue of the transposed convolution (upsample mode, Cout a power of two): column n of the
// accumulator is phase n / Cout, channel n % Cout. The warp's chunks are read from TMEM four per
// wait, the phase / channel of each chunk and its byte offset are computed once per unit, and
// the per-channel scale and bias (the e4m3 output scale folded in) come from shared memory as
// float4s. Rows map to input voxels; each chunk goes to the phase's output cell of that voxel.
template <int NCH, bool SPLITC>
__device__ void epilogue_up(const ConvParams& p, SmemCtl* ctl, int n_units) {
    const int lane = threadIdx.x & 31;
    const int wq = (threadIdx.x >> 5) & 3;
    const int half = ((threadIdx.x >> 5) - 2) >> 2;
    const uint32_t tbase = ctl->tmem_base;
    const uint32_t slot_cols = static_cast<uint32_t>(p.R * p.N_tile);
    const int Mtot = 128 * p.R;
    RowDecomp rd;
    rd.P2 = static_cast<uint32_t>(p.Hp * p.Wp);
    rd.Wp = static_cast<uint32_t>(p.Wp);
    rd.mP2 = ~0ull / rd.P2 + 1;
    rd.mWp = ~0ull / rd.Wp + 1;
    const uint32_t zmax = static_cast<uint32_t>(p.Dp - 2), ymax = static_cast<uint32_t>(p.Hp - 2),
                   xmax = static_cast<uint32_t>(p.Wp - 2);
    constexpr int kMy = SPLITC ? NCH / 2 : NCH;
    constexpr int kCs = SPLITC ? 2 : 1;
    const int c0 = SPLITC ? half : 0;
    const int rb = SPLITC ? 0 : half, rs = SPLITC ? 1 : 2;
    constexpr int kGrp = kMy <= 4 ? kMy : 4;  // chunks read from TMEM per wait
    const bool e4out = p.out_type == kOpE4M3;
    const int lc = __ffs(p.cout) - 1;  // log2(Cout)
    const int64_t oP2 = static_cast<int64_t>(p.oHp) * p.oWp;
    // factor along each axis and the bit of a phase index that holds each axis's parity
    const int um = p.up_mask;
    const int uz = (um & 4) ? 2 : 1, uy = (um & 2) ? 2 : 1, ux = (um & 1) ? 2 : 1;
    const int bx = 0, by = (um & 1) ? 1 : 0, bz = by + ((um & 2) ? 1 : 0);
    uint32_t j = 0;
    for (int unit = blockIdx.x; unit < n_units; unit += gridDim.x, ++j) {
        int b, mu, nt;
        unit_coords(p, unit, b, mu, nt);
        const int aslot = j % p.acc_slots;
        {
            FX_T0();
            if (!mbar_wait(smem_u32(&ctl->accf[aslot]), (j / p.acc_slots) & 1u, &ctl->abort, wait_limit(p))) {
                set_status(p.status, kStatusTimeoutAcc);
                ctl->abort = 1;
                return;
            }
            if (threadIdx.x == 64) FX_TADD(p, 5);
        }
        tc_fence_after();
        FX_T0();
        const int64_t q0 = p.row_begin + static_cast<int64_t>(mu) * Mtot;
        const int cbase = nt * p.N_tile;
        int32_t cofs[kMy];  // per chunk: its first channel
        int32_t boff[kMy];  // per chunk: byte offset of its cell from the voxel's phase-0 cell (< 2 GB)
#pragma unroll
        for (int c = 0; c < kMy; ++c) {
            const int n0 = cbase + (c0 + c * kCs) * 16;
            const int a = n0 >> lc, co0 = n0 - (a << lc);
            cofs[c] = co0;
            const int dz = uz == 2 ? (a >> bz) & 1 : 0, dy = uy == 2 ? (a >> by) & 1 : 0, dx = ux == 2 ? (a >> bx) & 1 : 0;
            const int64_t cell = dz * oP2 + dy * static_cast<int64_t>(p.oWp) + dx;
            boff[c] = static_cast<int32_t>(cell * 16 + static_cast<int64_t>(co0 / (e4out ? 16 : 8)) * p.out_group_stride);
        }
        for (int r = rb; r < p.R; r += rs) {
            const int64_t row = q0 + r * 128 + wq * 32 + lane;
            uint32_t z, y, x;
            rd.split(static_cast<uint32_t>(row), z, y, x);
            const bool valid = row < p.row_end && z >= 1 && z <= zmax && y >= 1 && y <= ymax && x >= 1 && x <= xmax;
            const uint32_t taddr =
                tbase + (static_cast<uint32_t>(wq * 32) << 16) + aslot * slot_cols + r * p.N_tile;
            uint8_t* ob = nullptr;
            if (valid)
                ob = p.out + static_cast<int64_t>(b) * p.out_batch_stride +
                     ((static_cast<int64_t>(uz * (z - 1) + 1) * p.oHp + (uy * (y - 1) + 1)) * p.oWp +
                      (ux * (x - 1) + 1)) * 16;
#pragma unroll
            for (int g0 = 0; g0 < kMy; g0 += kGrp) {
                uint32_t raw[kGrp][16];
#pragma unroll
                for (int c = 0; c < kGrp; ++c) tmem_ld16_nowait(taddr + (c0 + (g0 + c) * kCs) * 16, raw[c]);
                tmem_wait();
#pragma unroll
                for (int c = 0; c < kGrp; ++c) tmem_regs_ready(raw[c]);
                if (!valid) continue;
#pragma unroll
                for (int c = 0; c < kGrp; ++c) {
                    const int ci = g0 + c;
                    const float4* cs4 = reinterpret_cast<const float4*>(ctl->colscale + cofs[ci]);
                    const float4* bs4 = reinterpret_cast<const float4*>(ctl->bias + cofs[ci]);
                    float v[16];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 cs = cs4[q], bs = bs4[q];
                        v[4 * q + 0] = fmaf(__uint_as_float(raw[c][4 * q + 0]), cs.x, bs.x);
                        v[4 * q + 1] = fmaf(__uint_as_float(raw[c][4 * q + 1]), cs.y, bs.y);
                        v[4 * q + 2] = fmaf(__uint_as_float(raw[c][4 * q + 2]), cs.z, bs.z);
                        v[4 * q + 3] = fmaf(__uint_as_float(raw[c][4 * q + 3]), cs.w, bs.w);
                    }
                    if (p.amax) {
                        float mx = 0.f;
#pragma unroll
                        for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(v[i]));
                        if (e4out) mx /= p.out_qscale;
                        atomicMax(p.amax, __float_as_uint(mx));
                    }
                    uint8_t* o = ob + boff[ci];
                    if (e4out) {
                        uint4 w;
                        w.x = pack_e4m3x4(v[0], v[1], v[2], v[3]);
                        w.y = pack_e4m3x4(v[4], v[5], v[6], v[7]);
                        w.z = pack_e4m3x4(v[8], v[9], v[10], v[11]);
                        w.w = pack_e4m3x4(v[12], v[13], v[14], v[15]);
                        *reinterpret_cast<uint4*>(o) = w;
                    } else {
                        *reinterpret_cast<uint4*>(o) = pack_cell16(v, p.out_type);
                        *reinterpret_cast<uint4*>(o + p.out_group_stride) = pack_cell16(v + 8, p.out_type);
                    }
                }
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ctl->acce[aslot]));
        if (threadIdx.x == 64) {
            FX_TADD(p, 6);
            FX_TCNT(p, 8, 1);
        }
    }
}

// Epilogue of the x-tap fold (prenorm mode, Cout = 16 NC): a block's TMEM holds D0 | D1 | D2
// (N = 16 NC columns each); output row j = D0[j] + D1[j + 1] + D2[j + 2] for j < 126. Within a
// warp the row shifts are shuffles; the two rows that cross into the next lane quarter come
// through shared memory: every warp first publishes D1 of its lane 0 and D2 of its lanes 0 and 1,
// then the four warps of its half meet at an mbarrier (a bounded wait, like every wait of this
// kernel). The publish slots alternate between two parities so one meeting per M block suffices. The warp pair of a quarter splits the work
// like epilogue_loop (alternate M blocks, or alternate chunks when a unit has one M block).
template <int NC, bool SPLITC>
__device__ void epilogue_fold(const ConvParams& p, SmemCtl* ctl, float* xbuf, int n_units) {
    constexpr int N = NC * 16;
    const int lane = threadIdx.x & 31;
    const int wq = (threadIdx.x >> 5) & 3;
    const int half = ((threadIdx.x >> 5) - 2) >> 2;
    const uint32_t tbase = ctl->tmem_base;
    const uint32_t slot_cols = static_cast<uint32_t>(p.R * 3 * N);
    const int BR = p.block_rows;
    const int64_t Mtot = static_cast<int64_t>(BR) * p.R;
    RowDecomp rd;
    rd.P2 = static_cast<uint32_t>(p.Hp * p.Wp);
    rd.Wp = static_cast<uint32_t>(p.Wp);
    rd.mP2 = ~0ull / rd.P2 + 1;
    rd.mWp = ~0ull / rd.Wp + 1;
    const uint32_t zmax = static_cast<uint32_t>(p.Dp - 2), ymax = static_cast<uint32_t>(p.Hp - 2),
                   xmax = static_cast<uint32_t>(p.Wp - 2);
    const bool percol = p.col_scale != nullptr;
    const float acc_scale = p.acc_scale;
    constexpr int kMy = SPLITC ? NC / 2 : NC;
    constexpr int kCs = SPLITC ? 2 : 1;
    const int c0 = SPLITC ? half : 0;
    const int rb = SPLITC ? 0 : half, rs = SPLITC ? 1 : 2;
    constexpr bool kAccR = kMy == 1;
    float* xh = xbuf + half * (2 * 4 * 3 * N);  // [parity][quarter][D1 lane 0 | D2 lane 0 | D2 lane 1][N]
    uint32_t par = 0;
    uint32_t xph[2] = {0u, 0u};  // phase parity of xready[half][0 / 1]
    const int m = wq * 32 + lane;  // accumulator row of this thread
    uint32_t j = 0;
    for (int unit = blockIdx.x; unit < n_units; unit += gridDim.x, ++j) {
        int b, mu, nt;
        unit_coords(p, unit, b, mu, nt);
        const int aslot = j % p.acc_slots;
        {
            FX_T0();
            if (!mbar_wait(smem_u32(&ctl->accf[aslot]), (j / p.acc_slots) & 1u, &ctl->abort, wait_limit(p))) {
                set_status(p.status, kStatusTimeoutAcc);
                ctl->abort = 1;
                return;
            }
            if (threadIdx.x == 64) FX_TADD(p, 5);
        }
        tc_fence_after();
        FX_T0();
        const int64_t q0 = p.row_begin + static_cast<int64_t>(mu) * Mtot;
        float s1[kMy], s2[kMy];
        float r1[kAccR ? 1 : 1][16], r2[kAccR ? 1 : 1][16];
#pragma unroll
        for (int c = 0; c < kMy; ++c) s1[c] = s2[c] = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) r1[0][i] = r2[0][i] = 0.f;
        for (int r = rb; r < p.R; r += rs) {
            const int64_t row = q0 + static_cast<int64_t>(r) * BR + m;
            uint32_t z, y, x;
            rd.split(static_cast<uint32_t>(row), z, y, x);
            const bool valid = m < BR && row < p.row_end && z >= 1 && z <= zmax && y >= 1 && y <= ymax && x >= 1 &&
                               x <= xmax;
            const uint32_t taddr =
                tbase + (static_cast<uint32_t>(wq * 32) << 16) + aslot * slot_cols + static_cast<uint32_t>(r * 3 * N);
            float* xw = xh + (par * 4 + wq) * 3 * N;
            const float* xn = xh + (par * 4 + ((wq + 1) & 3)) * 3 * N;
            // publish the rows the previous lane quarter needs
#pragma unroll
            for (int i = 0; i < kMy; ++i) {
                const int cc = c0 + i * kCs;
                uint32_t u1[16], u2[16];
                tmem_ld16_nowait(taddr + N + cc * 16, u1);
                tmem_ld16_nowait(taddr + 2 * N + cc * 16, u2);
                tmem_wait();
                tmem_regs_ready(u1);
                tmem_regs_ready(u2);
                if (lane == 0) {
#pragma unroll
                    for (int t = 0; t < 16; t += 4) {
                        *reinterpret_cast<float4*>(xw + cc * 16 + t) =
                            make_float4(__uint_as_float(u1[t]), __uint_as_float(u1[t + 1]), __uint_as_float(u1[t + 2]),
                                        __uint_as_float(u1[t + 3]));
                        *reinterpret_cast<float4*>(xw + N + cc * 16 + t) =
                            make_float4(__uint_as_float(u2[t]), __uint_as_float(u2[t + 1]), __uint_as_float(u2[t + 2]),
                                        __uint_as_float(u2[t + 3]));
                    }
                } else if (lane == 1) {
#pragma unroll
                    for (int t = 0; t < 16; t += 4)
                        *reinterpret_cast<float4*>(xw + 2 * N + cc * 16 + t) =
                            make_float4(__uint_as_float(u2[t]), __uint_as_float(u2[t + 1]), __uint_as_float(u2[t + 2]),
                                        __uint_as_float(u2[t + 3]));
                }
            }
            __syncwarp();  // lane 1's publish is ordered before lane 0's arrive
            if (lane == 0) mbar_arrive(smem_u32(&ctl->xready[half][par]));
            if (!mbar_wait(smem_u32(&ctl->xready[half][par]), xph[par], &ctl->abort, wait_limit(p))) {
                set_status(p.status, kStatusTimeoutExchange);
                ctl->abort = 1;
                return;
            }
            xph[par] ^= 1u;
#pragma unroll
            for (int i = 0; i < kMy; ++i) {
                const int cc = c0 + i * kCs;
                uint32_t u0[16], u1[16], u2[16];
                tmem_ld16_nowait(taddr + cc * 16, u0);
                tmem_ld16_nowait(taddr + N + cc * 16, u1);
                tmem_ld16_nowait(taddr + 2 * N + cc * 16, u2);
                tmem_wait();
                tmem_regs_ready(u0);
                tmem_regs_ready(u1);
                tmem_regs_ready(u2);
                float a[16], bb[16];
#pragma unroll
                for (int t = 0; t < 16; ++t) {
                    a[t] = __shfl_down_sync(0xffffffffu, __uint_as_float(u1[t]), 1);
                    bb[t] = __shfl_down_sync(0xffffffffu, __uint_as_float(u2[t]), 2);
                }
                if (lane >= 30) {  // rows 31 / 30 of the quarter: D1, D2 of the next quarter's rows 0 / 1
                    const float* sa = xn + cc * 16;
                    const float* sb = xn + (lane == 31 ? 2 * N : N) + cc * 16;
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        if (lane == 31) a[t] = sa[t];
                        bb[t] = sb[t];
                    }
                }
                float v[16];
#pragma unroll
                for (int t = 0; t < 16; ++t) {
                    const float sc = percol ? ctl->colscale[cc * 16 + t] : acc_scale;
                    v[t] = (__uint_as_float(u0[t]) + a[t] + bb[t]) * sc;
                }
                if (valid) {
                    uint8_t* o = p.out + static_cast<int64_t>(b) * p.out_batch_stride + row * 16 +
                                 static_cast<int64_t>(cc * 2) * p.out_group_stride;
                    *reinterpret_cast<uint4*>(o) = pack_cell_f16_sat(v);
                    *reinterpret_cast<uint4*>(o + p.out_group_stride) = pack_cell_f16_sat(v + 8);
                }
                if constexpr (kAccR) {
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        const float w = valid ? v[t] : 0.f;
                        r1[0][t] += w;
                        r2[0][t] = fmaf(w, w, r2[0][t]);
                    }
                } else {
                    float q[16];
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        v[t] = valid ? v[t] : 0.f;
                        q[t] = v[t] * v[t];
                    }
                    s1[i] += warp_transpose_reduce16(v, lane);
                    s2[i] += warp_transpose_reduce16(q, lane);
                }
            }
            par ^= 1u;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ctl->acce[aslot]));
        if constexpr (kAccR) {
            s1[0] = warp_transpose_reduce16(r1[0], lane);
            s2[0] = warp_transpose_reduce16(r2[0], lane);
        }
        float* dst = p.stats +
                     ((static_cast<int64_t>(b) * p.n_units_m + mu) * p.stat_recs + half * 4 + wq) * p.stats_C * 2;
        if (lane < 16) {
#pragma unroll
            for (int c = 0; c < kMy; ++c) {
                const int ch = (c0 + c * kCs) * 16 + lane;
                *reinterpret_cast<float2*>(dst + ch * 2) = make_float2(s1[c], s2[c]);
                if (SPLITC) {
                    const int cho = ((c0 ^ 1) + c * kCs) * 16 + lane;
                    *reinterpret_cast<float2*>(dst + cho * 2) = make_float2(0.f, 0.f);
                }
            }
        }
        if (threadIdx.x == 64) {
            FX_TADD(p, 6);
            FX_TCNT(p, 8, 1);
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
            mbar_init(smem_u32(&ctl->acce[i]), kEpiWarps);
        }
        mbar_init(smem_u32(&ctl->drain), 1);
        mbar_init(smem_u32(&ctl->bres), 1);
        mbar_init(smem_u32(&ctl->never), 1);
        for (int h = 0; h < 2; ++h)
            for (int q = 0; q < 2; ++q) mbar_init(smem_u32(&ctl->xready[h][q]), 4);
        ctl->abort = 0;
        fence_mbar_init();
    }
    // per-channel dequant scale and bias tables (prenorm: by column; upsample: by channel)
    const int ncols = p.mode == kModeUpsample ? p.cout : p.stats_C;
    // upsample mode writes e4m3 cells as y * out_qscale: fold that factor into both tables
    const float osc = (p.mode == kModeUpsample && p.out_type == kOpE4M3) ? p.out_qscale : 1.f;
    for (int i = threadIdx.x; i < kMaxCols; i += blockDim.x) {
        ctl->colscale[i] = ((i < ncols && p.col_scale) ? p.col_scale[i] : 1.f) * osc;
        ctl->bias[i] = ((i < ncols && p.bias) ? p.bias[i] : 0.f) * osc;
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&ctl->tmem_base), p.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    (void)lane;
    // the allocation must lie inside the columns asked for (lane field 0, column + width <= 512)
    const uint32_t tb = ctl->tmem_base;
    const bool tmem_ok = (tb >> 16) == 0u && (tb & 0xFFFFu) + p.tmem_cols <= 512u;
    if (!tmem_ok) {
        if (threadIdx.x == 0) set_status(p.status, kStatusBadTmem);
    } else if (warp == 0) {
        producer_loop(p, smem, ctl, n_units);
    } else if (warp == 1 && p.zfold) {
        const bool f8 = p.optype == kOpE4M3;
        if (p.zplanes == 4) f8 ? mma_loop_z<true, 4>(p, smem, ctl, n_units) : mma_loop_z<false, 4>(p, smem, ctl, n_units);
        else f8 ? mma_loop_z<true, 2>(p, smem, ctl, n_units) : mma_loop_z<false, 2>(p, smem, ctl, n_units);
    } else if (warp == 1 && p.fold) {
        const bool f8 = p.optype == kOpE4M3;
        switch (p.R) {
            case 1: f8 ? mma_loop<1, true, false, true>(p, smem, ctl, n_units) : mma_loop<1, false, false, true>(p, smem, ctl, n_units); break;
            case 2: f8 ? mma_loop<2, true, false, true>(p, smem, ctl, n_units) : mma_loop<2, false, false, true>(p, smem, ctl, n_units); break;
            case 4: f8 ? mma_loop<4, true, false, true>(p, smem, ctl, n_units) : mma_loop<4, false, false, true>(p, smem, ctl, n_units); break;
            default: break;  // rejected on the host (launch_conv_tc)
        }
    } else if (warp == 1) {
        const bool f8 = p.optype == kOpE4M3, split = p.N_tile > 256;
        switch (p.R) {
            case 1:
                if (split) f8 ? mma_loop<1, true, true, false>(p, smem, ctl, n_units) : mma_loop<1, false, true, false>(p, smem, ctl, n_units);
                else f8 ? mma_loop<1, true, false, false>(p, smem, ctl, n_units) : mma_loop<1, false, false, false>(p, smem, ctl, n_units);
                break;
            case 2: f8 ? mma_loop<2, true, false, false>(p, smem, ctl, n_units) : mma_loop<2, false, false, false>(p, smem, ctl, n_units); break;
            case 4: f8 ? mma_loop<4, true, false, false>(p, smem, ctl, n_units) : mma_loop<4, false, false, false>(p, smem, ctl, n_units); break;
            case 8: f8 ? mma_loop<8, true, false, false>(p, smem, ctl, n_units) : mma_loop<8, false, false, false>(p, smem, ctl, n_units); break;
            default: break;  // rejected on the host (launch_conv_tc)
        }
    } else if (p.fold) {
        float* xbuf = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ctl) + sizeof(SmemCtl));
        const bool sc = p.R == 1;
        switch (p.N_tile / 48) {
            case 1: epilogue_fold<1, false>(p, ctl, xbuf, n_units); break;
            case 2: sc ? epilogue_fold<2, true>(p, ctl, xbuf, n_units) : epilogue_fold<2, false>(p, ctl, xbuf, n_units); break;
            case 4: sc ? epilogue_fold<4, true>(p, ctl, xbuf, n_units) : epilogue_fold<4, false>(p, ctl, xbuf, n_units); break;
            default: break;  // rejected on the host (launch_conv_tc)
        }
    } else if (p.mode == kModeUpsample && p.cout >= 16 && (p.cout & (p.cout - 1)) == 0 &&
               (static_cast<int64_t>(p.cout / 8) * p.out_group_stride +
                static_cast<int64_t>(p.oHp + 1) * p.oWp * 16) < (1ll << 31)) {  // 32-bit chunk offsets
        const bool sc = p.R == 1;
        switch (p.N_tile / 16) {
            case 2: sc ? epilogue_up<2, true>(p, ctl, n_units) : epilogue_up<2, false>(p, ctl, n_units); break;
            case 4: sc ? epilogue_up<4, true>(p, ctl, n_units) : epilogue_up<4, false>(p, ctl, n_units); break;
            case 8: sc ? epilogue_up<8, true>(p, ctl, n_units) : epilogue_up<8, false>(p, ctl, n_units); break;
            case 16: epilogue_up<16, true>(p, ctl, n_units); break;
            default: break;  // rejected on the host (launch_conv_tc)
        }
    } else {
        // split the chunks between the warp pair for one M block per unit, and for pre-norm tiles of
        // 32 / 64 columns (one / two chunks per warp and block: statistics summed in registers, the
        // TMEM reads of several blocks per wait)
        const bool sc = p.R == 1 || (p.mode == kModePrenorm && p.N_tile <= 64);  // (mirrored in launch_conv_tc)
        switch (p.N_tile / 16) {
            case 1: epilogue_loop<1, false>(p, ctl, n_units); break;
            case 2: sc ? epilogue_loop<2, true>(p, ctl, n_units) : epilogue_loop<2, false>(p, ctl, n_units); break;
            case 4: sc ? epilogue_loop<4, true>(p, ctl, n_units) : epilogue_loop<4, false>(p, ctl, n_units); break;
            case 8: sc ? epilogue_loop<8, true>(p, ctl, n_units) : epilogue_loop<8, false>(p, ctl, n_units); break;
            case 16: epilogue_loop<16, true>(p, ctl, n_units); break;   // N 256: always R = 1
            case 20: epilogue_loop<20, true>(p, ctl, n_units); break;   // N 320: always R = 1
            default: break;  // rejected on the host (launch_conv_tc)
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(ctl->tmem_base, p.tmem_cols);
    }
}

size_t conv_tc_ctl_bytes() { return sizeof(SmemCtl); }
size_t conv_tc_fold_bytes(int cout) { return static_cast<size_t>(2 * 2 * 4 * 3) * cout * sizeof(float); }

cudaError_t launch_conv_tc(const ConvParams& p, int grid, size_t smem_bytes, cudaStream_t stream) {
    // the dynamic shared memory limit is a per-device function attribute: set it once on every device
    // a launch comes to (threads driving several GPUs launch concurrently)
    static std::atomic<uint64_t> configured[4] = {};
    int dev = 0;
    if (cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return e;
    if (dev < 0 || dev >= 256) return cudaErrorInvalidDevice;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(configured[dev >> 6].load(std::memory_order_acquire) & bit)) {
        cudaError_t e =
            cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
        if (e != cudaSuccess) return e;
        configured[dev >> 6].fetch_or(bit, std::memory_order_acq_rel);
    }
    const int nch = p.N_tile / 16;
    if (!p.fold && (p.N_tile % 16 || !(nch == 1 || nch == 2 || nch == 4 || nch == 8 || nch == 16 || nch == 20)))
        return cudaErrorInvalidValue;
    if ((p.mode == kModeUpsample ? p.cout : p.stats_C) > kMaxCols) return cudaErrorInvalidValue;
    // four statistics records per unit only where the epilogue's warp pair splits the chunks
    if (p.mode == kModePrenorm &&
        !(p.stat_recs == kStatRecsPerUnit ||
          (p.stat_recs == kStatRecsPerUnit / 2 && !p.fold && p.N_tile >= 32 && (p.R == 1 || p.N_tile <= 64))))
        return cudaErrorInvalidValue;
    if (!(p.R == 1 || p.R == 2 || p.R == 4 || p.R == 8) || (p.N_tile > 256 && p.R != 1)) return cudaErrorInvalidValue;
    if (p.n_stages > kMaxStages || p.n_mmas > kMaxMmas) return cudaErrorInvalidValue;
    size_t need = static_cast<size_t>(p.n_pipe) * p.stage_bytes + sizeof(SmemCtl);
    if (p.fold) {
        const int nf = p.N_tile / 3;
        if (p.mode != kModePrenorm || p.N_tile % 48 || !(nf == 16 || nf == 32 || nf == 64) || p.stats_C != nf ||
            p.n_tiles != 1 || p.block_rows != 126 || !(p.R == 1 || p.R == 2 || p.R == 4) ||
            p.acc_slots * p.R * p.N_tile > static_cast<int>(p.tmem_cols))
            return cudaErrorInvalidValue;
        need += conv_tc_fold_bytes(nf);
    } else if (p.block_rows != 128) {
        return cudaErrorInvalidValue;
    }
    if (p.zfold) {
        if (p.fold || p.mode != kModePrenorm || p.n_tiles != 1 || !(p.R == 2 || p.R == 4 || p.R == 8) ||
            !(p.zplanes == 2 || p.zplanes == 4) || p.R != 2 * p.zplanes || p.zseg <= 0 || p.n_stages != p.zplanes + 2 || p.n_mmas <= 0 || p.bres_off % 128 || p.bres_bytes % 16 ||
            p.bres_bytes < 3 * p.n_mmas * p.N_tile * 32 || p.zkstride != p.N_tile * 16 ||
            p.N_tile * (p.zplanes < 3 ? p.zplanes : 3) > 256 || static_cast<size_t>(p.bres_off) < need ||
            p.acc_slots * p.R * p.N_tile > static_cast<int>(p.tmem_cols))
            return cudaErrorInvalidValue;
        need = static_cast<size_t>(p.bres_off) + p.bres_bytes;
    }
    if (smem_bytes < need || smem_bytes > 232448) return cudaErrorInvalidValue;
    count_launch();
    conv_tc_kernel<<<grid, kConvThreads, smem_bytes, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace fxk
