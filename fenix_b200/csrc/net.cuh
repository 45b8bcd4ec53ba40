// net.cuh — the plain 3D UNet (nnU-Net style: per stage 2 x [conv3 + InstanceNorm + LeakyReLU],
// stride-2 conv downsampling, ConvTranspose3d 2^3 upsampling, skip concat, 1x1x1 head) run on
// the B200 kernels, plus the sliding-window driver around it. Module semantics follow the
// reference's nets::ConvNormAct / ConvStack / Decoder (src/ml/nets/resenc_unet.hpp:35-52,
// 141-158, 197-239); the driver follows ml::predict_surface_filled (src/ml/infer.hpp:456-864).
#pragma once

#include "fenix_b200.h"
#include "conv_tc.cuh"
#include "eltwise.cuh"
#include "fxweights.hpp"
#include "program.hpp"

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

namespace fxk {
size_t conv_tc_ctl_bytes();
}

namespace fxh {

// Status code (values of fx_status) + message.
struct Status {
    int code = 0;
    std::string msg;
    bool ok() const { return code == 0; }
};
inline Status ok() { return {}; }
inline Status fail(int code, std::string m) { return {code, std::move(m)}; }
constexpr int kInvalid = 1, kNotFound = 2, kIo = 3, kDecode = 5, kUnsupported = 6, kInternal = 8;

Status cuda_status(cudaError_t e, const char* what);

// Padded group-plane tensor geometry (see conv_tc.cuh).
struct ActGeom {
    int D = 0, H = 0, W = 0;
    int64_t rows() const { return static_cast<int64_t>(D + 2) * (H + 2) * (W + 2); }
    int64_t gs() const { return rows() * 16; }
};

struct DevProgram {
    uint8_t* wpack = nullptr;
    float* colscale = nullptr;
    float* bias = nullptr;
    // prenorm layers: the epilogue scales every column by acc_scale; ratio[c] = colscale[c] /
    // acc_scale (null when 1) goes to the InstanceNorm statistics instead
    float acc_scale = 1.f;
    float* ratio = nullptr;
    Program host;
    int R = 1, N_tile = 0, acc_slots = 1, n_units_m = 0;
    uint32_t tmem_cols = 32;
    ActGeom rowspace;  // output grid (conv) or input grid (transposed conv)
    int optype = 0;    // fxk::OpType of the operands
    bool fold = false;     // x-tap fold (fxk::ConvParams::fold)
    bool zfold = false;    // z-plane fold (fxk::ConvParams::zfold)
    int zseg = 0;          // z-plane fold: units per plane
    int zplanes = 0;       // z-plane fold: planes per unit
    int block_rows = 128;
    bool built = false;
    size_t smem() const;
};

struct Layer {
    // kProj: a residual block's skip projection, 1x1x1 (stride 1) or AvgPool(2) + 1x1x1 as one
    // stride-2 program of 8 taps over the phase-split input with weights / 8
    enum Kind { kConv, kFirst, kUp, kProj } kind = kConv;
    std::string name;
    int Cin = 0, Cout = 0, stride = 1;
    // strided convs and transposed convs: the axes with factor 2 (bit 2 z, bit 1 y, bit 0 x). The
    // surface nets halve every axis (7); the layer-stack (ink) net halves y and x only in its
    // first strided stages (3).
    int smask = 0;
    int lin = 0, lout = 0;            // resolution levels of input and output
    std::vector<float> w;             // conv: [Cout][Cin][27]; up: [Cin][Cout][8]
    std::vector<float> b;             // up: bias (conv biases cancel inside InstanceNorm)
    std::vector<float> gamma, beta;   // InstanceNorm affine
    std::vector<float> wscale;        // fp8 per-output-channel weight scale (amax / 448)
    float in_scale = 1.f;             // fp8 per-tensor scale of the input activation
    bool keep16 = false;              // fp8 nets: precision schedule keeps this layer on 16-bit operands
    int idx = -1;                     // position in act_scales() order
    DevProgram prog[3];               // indexed by fxk::OpType: bf16, e4m3, f16
    float* d_gamma = nullptr;
    float* d_beta = nullptr;
    float* d_partials = nullptr;      // [Bmax][nrec][Cout][2]: per CTA (or per unit for the x fold)
    float* d_ss = nullptr;            // [Bmax][Cout][2]
    int nrec = 0;
    int64_t nrec_cap = 0;             // records per batch item that d_partials holds
    bool partials_dirty = false;      // a conv wrote d_partials and no statistics pass has cleared it
    const float* cur_ratio = nullptr; // ratio of the last prenorm launch (its statistics' scale)
};

// Compile one layer's program for operand type q (fxk::OpType) and upload it; gin/gout are
// the input and output grids. Device buffers are appended to `allocs` (owned by the caller).
Status build_layer_program(Layer& L, int q, ActGeom gin, ActGeom gout, int Bmax, int sm_count,
                           std::vector<void*>& allocs);
// Launch one layer. Stride-2 convs read the phase-split copy (gout geometry per phase); the
// prenorm mode writes L.d_partials and sets L.nrec.
// per_column: prenorm output scaled per column in the epilogue (exact pre-norm values, for
// callers that read them); otherwise by one factor, with the per-channel part in L.cur_ratio.
Status launch_layer(Layer& L, int q, ActGeom gin, ActGeom gout, const uint8_t* in_ptr, int64_t in_bs, int64_t in_gs,
                    uint8_t* out_ptr, int64_t out_bs, int64_t out_gs, int out_type, float out_qscale, unsigned* amax,
                    int nb, int sm_count, uint32_t* d_status, cudaStream_t s, bool per_column = false,
                    uint64_t wait_ns = 0, int stall_first_wait = 0);

// One BasicBlockD of a residual encoder (src/ml/nets/resenc_unet.hpp:103-135): indices into the
// net's encoder layers, the skip path and the scSE parameters.
struct ResBlock {
    int stage = 0;
    int c1 = -1, c2 = -1, proj = -1;  // conv1 (3x3x3, stride), conv2 (3x3x3), skip projection or -1
    int stride = 1;
    bool avgpool = false;             // stride 2 without projection: residual = AvgPool(2)(input)
    bool se = false;
    std::vector<float> cgate;         // cSE gate per channel: the block's GAP of IN(conv2) is the
                                      // norm's bias, so sigmoid(fc2(relu(fc1(beta)))) is a constant
    std::vector<float> sse_w;         // sSE conv 1x1 C -> 1
    float sse_b = 0.f;
    float* d_cgate = nullptr;
    float* d_sse_w = nullptr;
    int slot_x = 0, slot_h = 0;       // calibration amax slots of the block input / conv2 input
};

// Options of one sliding-window call beyond the tile grid (ml::InferOptions fields,
// src/ml/infer.hpp:38-103): the per-tile normalisation, the output crop, the constant-input tile
// skip and a caller's tile filter.
struct RunOpts {
    int norm = 0;               // 0 zscore, 1 pct_minmax, 2 unit255
    bool skip_constant = false; // tiles whose input voxels all hold one value are not run
    int (*filter)(int64_t z0, int64_t y0, int64_t x0, int64_t patch, void* user) = nullptr;
    void* filter_user = nullptr;
    // output crop in volume coordinates (core_ext <= 0: to the end of the volume). Tiles that do not
    // reach the core are not run; the accumulator covers the core along y and x (its z window is
    // predict_tiles' acc_z_origin / acc_dz).
    int64_t core_org[3] = {0, 0, 0};
    int64_t core_ext[3] = {0, 0, 0};
    // the volume is this many independent volumes of dz / stacks planes each, stacked along z:
    // tile starts and the blend run per stack, no tile crosses a stack boundary
    int stacks = 1;
};

class Net {
  public:
    ~Net();
    // tile = (z, y, x) extents of one tile; a cube for the surface nets
    Status create(const std::string& path, const int tile[3], int max_batch, int precision, int device);
    Status calibrate(const uint8_t* host_patches, int n);
    // Install per-layer input scales (act_scales() order) and build the e4m3 programs.
    Status set_act_scales(const float* scales, int n);
    // Forward nb tiles of a device volume at the given device tile origins. Head output:
    // Gaussian blend into acc (dims) and/or probabilities into prob ([nb][P^3]).
    // acc_z_shift / acc_dz: the accumulator is a window of acc_dz planes whose plane 0 is slab
    // plane -acc_z_shift (acc_dz < 0: the slab's own dz planes, shift 0).
    // d_tta: TTA member of each tile (null: none), tta_scale = 1 / members.
    Status forward(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, const fxk::TileOrigin* d_tiles, int nb,
                   int channel, int sigmoid, float* acc, float* prob, bool calib, cudaStream_t s,
                   int64_t acc_z_shift = 0, int64_t acc_dz = -1, const uint8_t* d_tta = nullptr,
                   float tta_scale = 1.f);
    // Tiles [tile_begin, tile_end) of the z-major grid over a (full_dz, dy, dx) volume. d_vol and
    // d_acc hold the z-slab [z_origin, z_origin + dz) of that volume; every tile of the range must
    // lie inside the slab.
    // With acc_dz >= 0, d_acc is a window of acc_dz planes starting at volume plane acc_z_origin
    // (contributions outside it are dropped), independent of the input slab.
    Status predict_tiles(const uint8_t* d_vol, int64_t dz, int64_t dy, int64_t dx, int64_t z_origin, int64_t full_dz,
                         fxk::TileDims tile, double overlap, int channel, int sigmoid, int batch, int64_t tile_begin,
                         int64_t tile_end, float* d_acc, cudaStream_t s, int64_t acc_z_origin = 0,
                         int64_t acc_dz = -1, int tta = 0, const RunOpts& ro = RunOpts{});
    // The normalisation forwards use (0 zscore, 1 pct_minmax, 2 unit255); calibration uses it too.
    void set_norm(int norm) { norm_ = norm; }
    // Device workspace for whole-volume calls: grown on demand, kept for the net's lifetime.
    Status workspace(size_t vol_bytes, size_t acc_bytes, size_t out_bytes, uint8_t** vol, float** acc, uint8_t** out);
    // A device buffer of at least n floats owned by the net (grown on demand; growing synchronises
    // the device, so a buffer still read by earlier asynchronous work is never freed under it).
    float* profile_buffer(size_t n);

    // the side of a cubic tile, 0 for an anisotropic one
    int patch() const { return tz_ == ty_ && ty_ == tx_ ? tz_ : 0; }
    fxk::TileDims tile() const { return {tz_, ty_, tx_}; }
    const std::vector<int>& stage_masks() const { return smask_; }
    int max_batch() const { return Bmax_; }
    int classes() const { return ncls_; }
    const std::vector<int>& features() const { return F_; }
    int precision() const { return prec_; }
    int t16() const { return prec_ == 0 ? 0 : 2; }  // 16-bit operand type: bf16 nets bf16, else f16
    int device() const { return dev_; }
    cudaStream_t stream() const { return stream_; }
    bool calibrated() const { return calibrated_; }
    std::vector<float> act_scales() const;
    // Precision schedule of an fp8 net, one entry per conv layer in act_scales() order:
    // fxk::kOpE4M3 (e4m3 where the layer can take it) or the 16-bit type. Layers that cannot run
    // e4m3 (the first conv, input channels not a multiple of 32) stay 16-bit whatever is asked.
    Status set_layer_precision(const int* q, int n);
    // Choose the precision schedule on n host calibration patches ([n][P][P][P] u8): the net's
    // 16-bit forward is the yardstick; every e4m3-capable layer is tried alone on e4m3 (agreement of
    // the 0.5-thresholded masks as Dice, and max |dp|), its conv time is measured on both operand
    // types, and layers are taken greedily by time saved per unit of squared Dice loss while the
    // summed squared losses stay within (1 - min_dice)^2 and each layer's max |dp| within max_abs
    // (<= 0: no bound). The chosen schedule is then run and layers are given back (last taken first)
    // until it meets both bounds. Calibrates the scales first if needed. Reports the schedule's Dice
    // and max |dp| against the 16-bit forward.
    Status calibrate_schedule(const uint8_t* host_patches, int n, double min_dice, double max_abs, double* dice,
                              double* maxabs);
    // The operand type each conv layer runs with (act_scales() order).
    std::vector<int> layer_precision() const;
    // Algorithmic FLOPs (2 x MACs) of one forward of one tile through each conv layer.
    std::vector<double> layer_flops() const;
    const Layer* layer_at(int i) const;
    // The device status word the kernels set on a bounded-wait timeout (0 = none); synchronises the
    // net's stream, then clears the word.
    Status take_device_status();

    // Per-conv-launch device timing with CUDA events on the launching stream (off by default).
    struct ProfileTotals {
        double conv_ms = 0, conv_flops = 0, fp8_flops = 0;
        int64_t conv_launches = 0;
    };
    void profile(bool on);
    // synchronises the recorded events; per-launch (ms, flops) pairs into `per` (up to cap)
    Status profile_read(ProfileTotals& out, double* per = nullptr, int cap = 0, std::vector<double>* per_layer = nullptr);

  private:
    struct ProfEv {
        cudaEvent_t a, b;
        double flops;
        int optype;
        int layer;
    };
    bool profile_ = false;
    std::vector<ProfEv> prof_;
    Status parse(const WeightMap& wm);
    // head: the head conv's prefix when it sits outside the decoder ("task_heads.<task>"); empty:
    // the decoder's seg_layers
    Status parse_resenc(const WeightMap& wm, const std::string& enc, const std::string& dec,
                        const std::string& head = "");
    Status alloc();
    Status build_layer(Layer& L, int q);
    Status run_conv(Layer& L, int q, const uint8_t* in_ptr, int64_t in_bs, int64_t in_gs, uint8_t* out_ptr,
                    int64_t out_bs, int64_t out_gs, int out_type, float out_qscale, unsigned* amax, int nb,
                    cudaStream_t s);
    Status finalize_in(Layer& L, int nb, cudaStream_t s);
    Status set_scales_from_amax();
    int layer_q(const Layer& L, bool calib) const;
    ActGeom level(int s) const { return lv_[static_cast<size_t>(s)]; }
    void* dalloc(size_t bytes);

    int tz_ = 0, ty_ = 0, tx_ = 0;  // tile extents
    int Bmax_ = 0, ncls_ = 2, prec_ = 0, dev_ = 0, S_ = 0, nconv_ = 2, sm_count_ = 148;
    std::vector<int> smask_;        // per stage: the axes its first conv halves (stage 0: none)
    std::vector<ActGeom> lv_;       // grid of each resolution level
    std::vector<int> F_;
    std::vector<Layer> enc_;  // S * nconv, stage-major
    std::vector<Layer> up_;   // S-1, index = level
    std::vector<Layer> dec_;  // (S-1) * nconv, index = level * nconv + i
    // residual encoder (stem + BasicBlockD stages) instead of the plain ConvStack encoder: enc_
    // holds the stem, then conv1, conv2, [projection] of every block in order
    bool resenc_ = false;
    std::vector<ResBlock> blocks_;
    std::vector<uint8_t*> h_, xf_, pnx_, res_;  // per level: conv2 input, f16 block input, projection pre-norm, pooled residual
    std::vector<float*> sg_;                    // per level: sSE gate
    int nslots_ = 0;                            // calibration amax slots
    std::vector<float> head_w_, head_b_;
    float* d_head_w_ = nullptr;
    float* d_head_b_ = nullptr;
    // activations (allocated at bf16 size; fp8 uses the first half of every group run)
    uint8_t* l0_ = nullptr;
    std::vector<uint8_t*> pn_, act_, cat_, ph_;
    unsigned long long* d_sums_ = nullptr;
    unsigned* d_hist_ = nullptr;  // [Bmax][256] u8 level counts (pct_minmax)
    float* d_luts_ = nullptr;     // [Bmax][256] per-tile normalisation tables
    int norm_ = 0;
    // accumulator window along y and x of the current sliding-window call (acc_dy_ <= 0: the volume)
    int64_t acc_y_shift_ = 0, acc_dy_ = 0, acc_x_shift_ = 0, acc_dx_ = 0;
    unsigned* d_amax_ = nullptr;  // calibration amax slots
    double* d_stat_work_ = nullptr;  // InstanceNorm slice sums [Bmax][kMaxStatSlices][Cmax][2]
    unsigned* d_stat_done_ = nullptr;  // slice counters [Bmax][Cmax / 32], zero between launches
    std::vector<float> amax_;
    float* d_gauss_ = nullptr;  // gaussian1d(tz), gaussian1d(ty), gaussian1d(tx) back to back
    uint32_t* d_status_ = nullptr;
    fxk::TileOrigin* d_tiles_ = nullptr;
    uint8_t* d_tta_ = nullptr;  // TTA member of each entry of d_tiles_
    int64_t d_tiles_cap_ = 0;
    uint8_t* ws_vol_ = nullptr;
    float* ws_acc_ = nullptr;
    uint8_t* ws_out_ = nullptr;
    size_t ws_vol_cap_ = 0, ws_acc_cap_ = 0, ws_out_cap_ = 0;
    float* ws_prof_ = nullptr;
    size_t ws_prof_cap_ = 0;
    cudaStream_t stream_ = nullptr;
    bool calibrated_ = false;
    std::vector<void*> allocs_;
};

}  // namespace fxh

// The opaque handle of include/fenix_b200.h.
struct fx_net {
    fxh::Net net;
};

namespace fxh {
// fx_infer_opts -> the driver's per-call options, and the output crop box it asks for (capi.cu).
RunOpts run_opts(const fx_infer_opts* o);
// The call's tile: opts.tile, or the cube of side opts.patch (divisible by 64); sets the error on failure.
fx_status opts_tile(const fx_infer_opts* o, fxk::TileDims* t);
void crop_box(const fx_infer_opts* o, const int64_t d[3], int64_t co[3], int64_t ce[3]);
// fx_predict_volume's device part (capi.cu), shared with the .fxvol entry points.
// Runs on stream s (null: the net's stream); sync = wait for it before returning.
fx_status predict_resident(fx_net* n, const uint8_t* d_vol, int64_t dz, int64_t dy, int64_t dx,
                           const fx_infer_opts* o, float* d_acc, float* d_prob, uint8_t* d_u8,
                           cudaStream_t s = nullptr, bool sync = true);
}  // namespace fxh
