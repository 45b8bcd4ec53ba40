// eltwise.cuh — the HBM-bound kernels around the convolutions: per-tile z-score normalise of
// the gathered u8 patch, InstanceNorm statistics finalise, normalise + LeakyReLU + requantise
// into the consumers' layouts, the fused 1x1x1 head + softmax/sigmoid + Gaussian blend, and the
// accumulator -> probability / u8 finalise.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace fxk {

// A view of one tensor in the padded group-plane layout (see conv_tc.cuh).
struct GridGeom {
    int32_t D, H, W;  // interior extents; padded extents are +2
};

struct TileOrigin {
    int64_t z0, y0, x0;
};

// Extents of one tile along z, y, x (the surface nets use cubes; the layer-stack ink net 64 x 256 x 256).
struct TileDims {
    int32_t z, y, x;
    __host__ __device__ int64_t count() const { return static_cast<int64_t>(z) * y * x; }
};

// ---- tiler ----------------------------------------------------------------------------------
// Integer sum and sum of squares of every tile's P^3 u8 voxels (edge-clamped reads), into
// sums[2*b + {0,1}] (exact; the caller zeroes `sums`), and with `hist` the count of each u8 level
// per tile, hist[256*b + v] (caller-zeroed).
cudaError_t launch_tile_sums(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, const TileOrigin* tiles,
                             int ntiles, TileDims P, unsigned long long* sums, cudaStream_t s, unsigned* hist = nullptr);
// Per-tile normalisation table of the 256 u8 levels, luts[256*b + v], for norm 0 zscore (from the
// sums), 1 pct_minmax (from the histogram), 2 unit255 (src/ml/infer.hpp:107-134, 350-385); with
// const_flag, 1 for each tile whose voxels all hold one value.
cudaError_t launch_tile_lut(const unsigned long long* sums, const unsigned* hist, int ntiles, int64_t n, int norm,
                            float* luts, uint8_t* const_flag, cudaStream_t s);
// Writes the first conv's input for every tile: the normalised values at x-1, x, x+1 (zero outside
// the tile). Normalisation goes through a 256-entry table per tile: luts[256*b ..] when given
// (launch_tile_lut), else the z-score table built here from `sums` with the reference's
// double-precision expression, so the normalised value of each u8 level is the same float the
// reference computes.
// `l0_type` is the first conv's operand type (kOpBF16 or kOpF16); l0 (may be null) receives its
// two input groups, l0_group_stride bytes apart (first_layer_cells: the value as hi + lo terms).
// tta (one byte per tile, or null): octahedral test-time-augmentation member of each tile; the
// tile is written in that member's frame (see tta_source).
cudaError_t launch_tile_norm(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, const TileOrigin* tiles,
                             int ntiles, TileDims P, const unsigned long long* sums, uint8_t* l0, int64_t l0_batch_stride,
                             int64_t l0_group_stride, int l0_type, float* f32_out, cudaStream_t s,
                             const uint8_t* tta = nullptr, const float* luts = nullptr);

// Octahedral TTA (src/ml/infer.hpp:346, 393-441): member m of the first N of 48 uses the axis
// permutation perms[m / 8] and flips the transformed frame's axes in the bits of m % 8 (bit 0 z,
// bit 1 y, bit 2 x). Voxel a of the member's frame is voxel o of the tile with
// o[perm[d]] = (flip_d ? P - 1 - a[d] : a[d]); the network's output at a belongs to o.
constexpr int kTtaMaxMembers = 48;
__host__ __device__ inline void tta_source(int m, int P, int a0, int a1, int a2, int& o0, int& o1, int& o2) {
    const int perm[6][3] = {{0, 1, 2}, {0, 2, 1}, {1, 0, 2}, {1, 2, 0}, {2, 0, 1}, {2, 1, 0}};
    const int pi = m >> 3, fm = m & 7;
    const int a[3] = {(fm & 1) ? P - 1 - a0 : a0, (fm & 2) ? P - 1 - a1 : a1, (fm & 4) ? P - 1 - a2 : a2};
    int o[3];
    o[perm[pi][0]] = a[0];
    o[perm[pi][1]] = a[1];
    o[perm[pi][2]] = a[2];
    o0 = o[0];
    o1 = o[1];
    o2 = o[2];
}

// ---- InstanceNorm ----------------------------------------------------------------------------
// partials [B][nrec][C][2] -> ss [B][C][2] = {scale, shift} with scale = gamma * rstd and
// shift = beta - mean * scale over `count` voxels. work holds B * kMaxStatSlices * C * 2 doubles;
// done holds B * ceil(C / 32) counters that are zero before the first launch (each launch leaves
// them zero). Launches sharing work/done must be stream-ordered. ratio (per channel, or null):
// the records hold each channel's values divided by ratio[c] (see in_stats_kernel). The records
// read are left at zero.
constexpr int kMaxStatSlices = 128;
cudaError_t launch_in_finalize(float* partials, int B, int nrec, int C, double count, const float* gamma,
                               const float* beta, const float* ratio, float eps, double* work, unsigned* done,
                               float* ss, cudaStream_t s);

struct NormDest {
    uint8_t* ptr;          // group 0 of the written slice, batch 0 (null = unused)
    int64_t batch_stride;  // bytes
    int64_t group_stride;  // bytes
    int32_t dtype;         // OpType of the written cells (e4m3 values are y * qscale)
    float qscale;
    int32_t phase;         // != 0: write the stride-2 phase-split copy over the axes of this mask
                           // (bit 2 z, bit 1 y, bit 0 x; one parity sub-volume per phase)
    int32_t pHp, pWp;      // phase sub-volume padded H, W (= output grid of the stride-2 conv)
    int64_t phase_stride;  // bytes between parity sub-volumes
};

// Checkpoint snapshot of a non-negative f32 accumulator: *max_bits = the float bits of max(acc)
// (atomicMax on the bits, caller-zeroed), and q[i] = (u16)(acc[i] * inv + 0.5f) with the multiply
// and the add rounded separately (src/ml/infer.hpp:177-182).
cudaError_t launch_acc_max(const float* acc, int64_t n, unsigned* max_bits, cudaStream_t s);
cudaError_t launch_acc_quant_u16(const float* acc, int64_t n, float inv, uint16_t* q, cudaStream_t s);

// y = leaky_relu(x * scale[c] + shift[c], slope) over the interior of an f16 pre-norm tensor,
// written to up to two destinations; optionally records max |y| into *amax (float bits).
cudaError_t launch_norm_act(const uint8_t* pre, int64_t pre_batch_stride, int64_t pre_group_stride, GridGeom g,
                            int C, int B, const float* ss, float slope, NormDest d0, NormDest d1, unsigned* amax,
                            cudaStream_t s);

// ---- residual encoder blocks (src/ml/nets/resenc_unet.hpp:103-135) ---------------------------
// Output of one BasicBlockD: y = leaky(out * (cgate[c] + sgate[v]) + res), out = the second conv's
// pre-norm x * ss[c].x + ss[c].y (InstanceNorm, no activation). Without scSE, cgate = 1 and
// sgate = 0 (pass null for both). res is the skip path: InstanceNorm of a projection's pre-norm
// output (res_ss non-null) or an f16 tensor (identity or average-pooled input) taken as is. All
// tensors are f16 padded group planes over the block's output grid; y goes to up to three
// destinations in their operand types. C % 16 == 0.
struct BlockOut {
    const uint8_t* pre;
    int64_t pre_bs, pre_gs;
    const float* ss;       // [B][C][2]
    const float* cgate;    // [C] or null
    const float* sgate;    // [B][D][H][W] f32 or null
    const uint8_t* res;
    int64_t res_bs, res_gs;
    const float* res_ss;   // [B][C][2] or null
    float slope;
    NormDest d[3];
    unsigned* amax;        // max |y| (float bits) or null
    GridGeom g;
    int32_t C, B;
};
cudaError_t launch_block_out(const BlockOut& p, cudaStream_t s);

// sgate[b][v] = sigmoid(sum_c w[c] * (pre[c] * ss[c].x + ss[c].y) + bias): the spatial squeeze-
// excitation gate (sSE conv 1x1 C -> 1) of the normalised second conv of a block.
cudaError_t launch_sse_gate(const uint8_t* pre, int64_t pre_bs, int64_t pre_gs, const float* ss, const float* w,
                            float bias, GridGeom g, int C, int B, float* sgate, cudaStream_t s);

// dst = AvgPool3d(2, stride 2) of an f16 padded group-plane tensor over grid gin into grid
// gout = gin / 2 (f16, same channel groups; the zero border of dst is left untouched).
cudaError_t launch_avgpool2_f16(const uint8_t* src, int64_t src_bs, int64_t src_gs, GridGeom gin, uint8_t* dst,
                                int64_t dst_bs, int64_t dst_gs, int groups, int B, cudaStream_t s);

// Last decoder layer: normalise + LeakyReLU, 1x1x1 head (ncls <= 2), softmax channel `channel`
// (or sigmoid of channel 0), NaN -> 0 / +inf -> 1, then Gaussian-blend into the volume
// accumulator at each tile's origin (acc may be null) and/or store the tile probability
// (prob may be null, [B][P^3] f32).
struct HeadParams {
    const uint8_t* pre;
    int64_t pre_batch_stride, pre_group_stride;
    int32_t Pz, Py, Px, C, B, ncls, channel, sigmoid;  // tile extents; TTA members need a cube
    const float* ss;     // [B][C][2]
    float slope;
    const float* wh;     // [ncls][C]
    const float* bh;     // [ncls]
    const float* gz;     // gaussian1d(Pz), gaussian1d(Py), gaussian1d(Px)
    const float* gy;
    const float* gx;
    const TileOrigin* tiles;
    const uint8_t* tta;  // TTA member of each tile (null: none); the output at a goes to tta_source(a)
    float tta_scale;     // 1 / members (the blend adds the members' mean)
    float* acc;          // accumulator planes or null (see acc_z_shift)
    int64_t dz, dy, dx;  // volume extents the tile origins refer to (voxels at z >= dz are skipped)
    // accumulator plane of volume plane z is z + acc_z_shift; planes outside [0, acc_dz) are not
    // written (a sliding window over a longer volume). acc_dz = dz, shift 0: the whole volume.
    int64_t acc_z_shift, acc_dz;
    // the same along y and x (an output crop): accumulator row y + acc_y_shift of acc_dy rows, column
    // x + acc_x_shift of acc_dx; acc_dy / acc_dx <= 0 mean the volume's dy / dx with shift 0
    int64_t acc_y_shift, acc_dy, acc_x_shift, acc_dx;
    float* prob;         // [B][P^3] or null
};
cudaError_t launch_head_blend(const HeadParams& h, cudaStream_t s);

// acc[z + acc_z_shift][y][x] += (gz * gy) * gx * p over one P^3 tile of probabilities at volume
// origin (z0, y0, x0) (the reference's scatter, src/ml/global_accum.hpp:79-116): voxels outside
// [0, dz) x [0, dy) x [0, dx), below plane z_floor, or outside the window [0, acc_dz) are skipped.
cudaError_t launch_scatter_tile(const float* prob, int P, int64_t z0, int64_t y0, int64_t x0, int64_t dz, int64_t dy,
                                int64_t dx, int64_t z_floor, const float* gauss, float* acc, int64_t acc_z_shift,
                                int64_t acc_dz, cudaStream_t s);

// acc / (Wz[z]*Wy[y]*Wx[x]) where the weight is > 0 (the reference's normalize), then
// u8 = (u8)(clamp(p, 0, 1) * 255 + 0.5), for planes [z_begin, z_end) of acc; the outputs hold
// just those planes (output plane 0 = plane z_begin). Either output may be null.
cudaError_t launch_accum_finalize(const float* acc, int64_t dz, int64_t dy, int64_t dx, int64_t z_begin,
                                  int64_t z_end, const float* Wz, const float* Wy, const float* Wx, float* prob,
                                  uint8_t* u8, cudaStream_t s);

cudaError_t launch_zero(void* p, size_t bytes, cudaStream_t s);
// dst[i] += src[i] (f32, n elements): folds another rank's accumulator band into this one.
cudaError_t launch_accum_add(float* dst, const float* src, int64_t n, cudaStream_t s);
cudaError_t launch_prob_compare(const float* a, const float* b, int64_t n, unsigned long long* stats,
                                unsigned* maxabs, cudaStream_t s);

}  // namespace fxk
