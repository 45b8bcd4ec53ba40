// pack.cuh — layout conversions between f32 NCDHW tensors and the padded group-plane layout,
// used by the per-op C entry points (parity tests, custom drivers) and by calibration.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace fxk {

// f32 [B][C][D][H][W] -> padded group planes of OpType `dtype` (e4m3 values are x*qscale). With
// `phase` != 0, writes the stride-2 phase-split copy over the axes of that mask (bit 2 z, bit 1 y,
// bit 0 x; sub-volume padded dims pHp x pWp, `phase_stride` bytes apart). Channels >= C inside the last group are written as zero.
cudaError_t launch_pack(const float* x, int B, int C, int D, int H, int W, uint8_t* out, int64_t batch_stride,
                        int64_t group_stride, int dtype, float qscale, int phase, int pHp, int pWp,
                        int64_t phase_stride, cudaStream_t s);
// f32 [B][1][D][H][W] -> the first layer's two x-folded 16-bit groups (first_layer_cells),
// group_stride bytes apart.
cudaError_t launch_pack_first(const float* x, int B, int D, int H, int W, uint8_t* out, int64_t batch_stride,
                              int64_t group_stride, int dtype, cudaStream_t s);
// padded group planes of OpType `dtype` -> f32 [B][C][D][H][W] (e4m3 values times `scale`).
cudaError_t launch_unpack(const uint8_t* in, int64_t batch_stride, int64_t group_stride, int dtype, float scale, int B,
                          int C, int D, int H, int W, float* y, cudaStream_t s);
// max |x| over n floats into *amax (float bits; caller zeroes).
cudaError_t launch_absmax(const float* x, int64_t n, unsigned* amax, cudaStream_t s);

}  // namespace fxk
