// conv_tc.cuh — the one tensor-core kernel behind every convolution of the UNet forward
// (3x3x3 stride 1, 3x3x3 stride 2, the 1-channel first layer, and the 2x2x2 stride-2
// transposed conv).
//
// Activation layout ("padded group planes"): a tensor of C channels over D x H x W voxels is
// stored as [batch][group][D+2][H+2][W+2][16 bytes], one group = 16 bytes of channels
// (8 bf16 or 16 e4m3), with a one-voxel zero border. Flattening (z, y, x) of one group gives a
// 1-D array of 16-byte "rows"; a 3x3x3 stride-1 conv is then a sum over 27 row shifts, and the
// A operand of every tap is a contiguous run of rows. The tcgen05 K-major no-swizzle smem
// layout keeps rows 16 B apart (SBO = 128 B), so a tap's A tile is just a descriptor whose start
// address is shifted by (tap offset x 16 B) inside one staged window — no im2col and no halo
// bookkeeping in the kernel. Stride-2 convs read a phase-split copy of their input (8 parity
// sub-volumes with the output's padded geometry), which turns the strided taps into row
// shifts as well.
//
// x-tap fold (3x3x3 stride 1, Cout <= 64): the program lists the 9 (kz, ky) taps with the A tile
// starting one row early, and each program MMA becomes three MMAs of N = Cout that share its A
// tile through the A collector (read from shared memory once) and accumulate x taps 0, 1, 2 into
// three accumulators D0, D1, D2 of the same M block. Output row j of the block is
// D0[j] + D1[j + 1] + D2[j + 2], so a block yields 126 output rows; the epilogue does the row
// shifts across lanes (shuffles, and shared memory across the warps' lane quarters).
//
// z-plane fold (3x3x3 stride 1): a unit's M blocks are S adjacent 128-row (y, x) segments in
// `zplanes` consecutive z planes, so output block (segment, r) and tap kz read input plane
// z0 + r + kz - 1: the A tile of input plane j (shift ky, kx) feeds blocks j, j-1, j-2 of its
// segment with taps kz = 0, 1, 2. The three taps' weights are consecutive rows of B and the
// planes of a segment sit at descending TMEM columns, so that is ONE MMA of N = 3 Cout (fewer at
// the first and last planes): one A read from shared memory and one issue for up to three
// accumulators, unshifted. Stages are input-plane windows; the 27 taps' weights stay resident in
// shared memory.
//
// The host compiles each layer into a small "program": a list of pipeline stages (one bulk
// copy of a window of rows for a range of groups + the matching packed weight block) and, per
// stage, the list of MMAs (A offset, K-half stride, B offset). The kernel is persistent and
// warp specialised: warp 0 issues the bulk copies, warp 1 issues tcgen05.mma from one thread
// and owns the TMEM allocation, warps 2..9 drain the TMEM accumulators (epilogue).
#pragma once

#include <cstddef>
#include <cstdint>

#include "optype.cuh"

namespace fxk {

constexpr int kConvThreads = 320;  // warp 0 producer, warp 1 MMA issuer, warps 2..9 epilogue
constexpr int kEpiWarps = 8;        // two per TMEM lane quarter, splitting the M blocks of a unit
// InstanceNorm partial records per CTA run (per work unit for the x-fold epilogue): one per
// epilogue warp, or half of that when the warp pair of a lane quarter shares one.
constexpr int kStatRecsPerUnit = kEpiWarps;
constexpr int kMaxSrc = 8;

struct ConvStage {
    int32_t src;        // source array index
    int32_t row_off;    // first window row relative to the unit's first output row
    int32_t rows;       // window length in rows
    int32_t g0, ng;     // group range copied
    int32_t b_off;      // byte offset of the packed B block (within one N tile's weights)
    int32_t b_bytes;
    int32_t mma_begin, mma_count;
};

// One MMA of a stage, pre-packed into the low words of its smem descriptors (16-byte units):
//   a = (lbo >> 4) << 16 | (A offset in the stage >> 4), b = B offset in the stage >> 4.
struct ConvMma {
    uint32_t a;
    uint32_t b;
};

constexpr int kMaxStages = 320;   // program capacity (kept in the kernel's parameter space)
constexpr int kMaxMmas = 1536;

struct ConvSrc {
    const uint8_t* ptr;    // row 0 of group 0 of batch item 0
    int64_t batch_stride;  // bytes
    int64_t group_stride;  // bytes
    int64_t rows;          // rows that exist per (batch, group)
};

enum ConvMode : int32_t {
    kModePrenorm = 0,  // store f16 pre-norm output, emit per-channel sum / sum of squares
    kModeUpsample = 1, // transposed conv: + bias, scatter 8 phases into the 2x finer grid
};

// Shared-memory bytes of the fold epilogue's row exchange for Cout output channels.
size_t conv_tc_fold_bytes(int cout);

struct ConvParams {
    ConvSrc src[kMaxSrc];
    const uint8_t* wpack;  // packed B blocks of N tile 0; tile t starts at + t * wtile_bytes
    int64_t wtile_bytes;
    int32_t n_stages;
    int32_t n_mmas;
    int32_t optype;  // OpType of both operands: bf16 / f16 (kind::f16) or e4m3 (kind::f8f6f4)

    // output-row space of one batch item: the padded geometry rows are indexed in
    int32_t batch;
    int32_t Dp, Hp, Wp;          // padded extents of the row space
    int64_t row_begin, row_end;  // rows computed per batch item
    int32_t R;                   // M blocks (of 128 accumulator rows) per work unit
    int32_t block_rows;          // output rows advanced per M block: 128, or 126 with fold
    int32_t fold;                // 1: the three x taps share each A tile (see below)
    int32_t zfold;               // 1: z-plane fold — the R blocks of a unit are one z plane apart
    int32_t zseg;                // z-plane fold: units per plane (each S adjacent 128-row segments)
    int32_t zplanes;             // z-plane fold: planes per unit; R = zplanes x S blocks
    int32_t zkstride;            // z-plane fold: bytes between the resident weight rows of kz and kz + 1
    int32_t bres_off, bres_bytes;  // z-plane fold: resident weights in shared memory (offset, size)
    int32_t n_units_m;           // ceil((row_end - row_begin) / (block_rows R))
    int32_t n_tiles;             // N tiles
    int32_t N_tile;              // accumulator columns per tile (multiple of 16)
    int32_t acc_slots;           // accumulator buffers in TMEM (1 or 2)
    uint32_t tmem_cols;          // power of two >= acc_slots * R * N_tile
    int32_t n_pipe;              // smem pipeline depth
    int32_t stage_bytes;         // bytes per pipeline stage
    int32_t stage_a_bytes;       // B block offset within a stage

    // epilogue
    int32_t mode;
    const float* col_scale;  // per output channel multiplier (fp8 dequant) or null
    float acc_scale;         // prenorm mode without col_scale: one multiplier for every column
    const float* bias;       // per output channel bias (upsample mode) or null
    uint8_t* out;            // output tensor, group 0 of the written channel slice, batch 0
    int64_t out_batch_stride, out_group_stride;  // bytes
    int32_t out_type;        // upsample mode: OpType of the written cells (e4m3 scaled by out_qscale)
    int32_t up_mask;         // upsample mode: the axes doubled (bit 2 z, bit 1 y, bit 0 x); the output
                             // phases (N_tile / cout of them) enumerate their parities in z, y, x order
    float out_qscale;
    int32_t cout;            // upsample mode: channels per phase
    int32_t oHp, oWp;        // upsample mode: padded H, W of the output grid
    unsigned* amax;          // upsample mode: max |output| (float bits) when non-null
    float* stats;            // prenorm mode: partial sums [batch][gridDim.x][stat_recs][C][2], which
                             // the epilogue ADDS into (zero before the launch); the x-fold epilogue
                             // writes [batch][n_units_m][stat_recs][C][2] instead
    int32_t stats_C;         // channels per stats record (= n_tiles * N_tile)
    int32_t stat_recs;       // prenorm mode: records per CTA (per unit for the x fold): kStatRecsPerUnit,
                             // or half of it when the epilogue's warp pair splits the chunks
                             // (N_tile >= 32 and R == 1 or N_tile <= 64, no x fold)
    uint32_t* status;
    uint64_t wait_ns;            // limit of every barrier wait in ns; 0 = the default (2 s)
    int32_t stall_first_wait;    // failure self-test only (fx_selftest_wait_timeout): the MMA warp's
                                 // first stage wait is on a barrier nothing arrives at, so it times
                                 // out and the launch ends with kStatusTimeoutFull
    unsigned long long* trace;  // per-role cycle counters (kernel built with FX_CONV_TRACE), or null
    // The program itself travels in the parameter space: warp-uniform indexed loads of it land in
    // uniform registers, so issuing an MMA costs a few uniform adds.
    ConvStage stages[kMaxStages];
    ConvMma mmas[kMaxMmas];
};

}  // namespace fxk
