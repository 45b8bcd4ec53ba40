/* fenix_b200.h — C ABI of the B200 (sm_100a) surface-prediction inference library.
 *
 * Plain C types only: pointers, sizes, enums. No exception crosses this boundary; every call
 * returns an fx_status (1:1 with the reference's fenix::Errc, src/core/error.hpp:19-29) and the
 * message of the last failure on the calling thread is available from fx_last_error().
 *
 * Which reference interface each entry point replaces:
 *   fx_net_create / fx_net_destroy  — building nets::ResEncUNet-style modules + load_fxweights /
 *                                     load_into (src/ml/inference.cpp:668-711,
 *                                     src/ml/weights.hpp:63-142), the TrtNet/AotiNet adapters'
 *                                     static batch/patch/classes (src/ml/trt_engine.hpp:35-106)
 *   fx_net_calibrate                — fp8 static calibration (tools/ml-export/fp8_forward.py:88-127)
 *   fx_net_set_norm                 — the stage's input normalisation for calibration and
 *                                     fx_net_forward (src/ml/inference.cpp:898-908, 721-740)
 *   fx_net_forward                  — the operator concept net->forward(x) followed by the
 *                                     softmax/sigmoid channel select + nan_to_num
 *                                     (src/ml/infer.hpp:760-767, src/ml/inference.cpp:226-233)
 *   fx_predict_volume               — ml::predict_surface_filled over a dense u8 volume
 *                                     (src/ml/infer.hpp:456-864) plus the u8 encode of
 *                                     run_predict_core (src/ml/inference.cpp:309-351)
 *   fx_tile_starts / fx_gaussian1d / fx_weight_profile
 *                                   — src/ml/tiling.hpp:16-42, src/ml/infer.hpp:499-509,
 *                                     src/ml/global_accum.hpp:29-35
 *   fx_norm_tiles                   — the dense u8 filler + detail::norm_patch (zscore)
 *                                     (src/ml/inference.cpp:309-321, src/ml/infer.hpp:350-385)
 *   fx_conv3d / fx_conv_transpose2  — one ConvNormAct conv / nn::ConvTranspose3d
 *                                     (src/ml/nets/resenc_unet.hpp:35-52, 211)
 *   fx_accum_finalize               — normalize() + u8 quantise (src/ml/infer.hpp:510-521,
 *                                     src/ml/global_accum.hpp:123-152)
 *   fx_gaccum_*                     — ml::GlobalAccum: global-grid accumulator, z-sweep
 *                                     finalize_rows_below, resume floor
 *                                     (src/ml/global_accum.hpp:37-198), and a tile row of
 *                                     predict-scroll's global mode (src/ml/inference.cpp:1282-1372)
 *   fx_fxvol_*                      — codec::VolumeArchive, the .fxvol v5 container
 *                                     (src/codec/archive.hpp:132-1217) with LOD-0 reads and
 *                                     write_volume encoded / decoded on the device
 *   fx_fxvol_encode_tiles / _decode_tiles
 *                                   — codec::encode_tile_dct / decode_tile_dct with bpa = 4
 *                                     (src/codec/dct_block.hpp:318-588)
 *   fx_predict_fxvol                — the predict-surface command over archives: .fxvol input
 *                                     read (src/ml/inference.cpp:540-567), prediction, u8 q=32
 *                                     .fxvol output (src/ml/inference.cpp:333-355)
 */
#ifndef FENIX_B200_H
#define FENIX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum fx_status {
    FX_OK = 0,
    FX_INVALID_ARGUMENT = 1,
    FX_NOT_FOUND = 2,
    FX_IO_ERROR = 3,
    FX_FETCH_FAILED = 4,
    FX_DECODE_ERROR = 5,
    FX_UNSUPPORTED = 6,
    FX_UNIMPLEMENTED = 7,
    FX_INTERNAL = 8
} fx_status;

/* Operand precision of the tensor-core convolutions (f32 accumulate in every case):
 * bf16 and f16 run tcgen05 kind::f16, fp8 runs kind::f8f6f4 with e4m3 activations (per-tensor
 * scale) and e4m3 weights (per-output-channel scale); in an fp8 net the first conv and any conv
 * whose input channels are not a multiple of 32 use f16. */
typedef enum fx_precision { FX_PREC_BF16 = 0, FX_PREC_FP8 = 1, FX_PREC_F16 = 2 } fx_precision;

/* Per-tile normalisation of the u8 input (src/ml/infer.hpp:107-134, 350-385 norm_patch). */
typedef enum fx_norm { FX_NORM_ZSCORE = 0, FX_NORM_PCT_MINMAX = 1, FX_NORM_UNIT255 = 2 } fx_norm;

/* A caller's tile filter (InferOptions::tile_filter, src/ml/infer.hpp:102): nonzero = run the
 * tile at (z0, y0, x0) of side `patch` (input coordinates). Called on the calling thread. */
typedef int (*fx_tile_filter_fn)(int64_t z0, int64_t y0, int64_t x0, int64_t patch, void* user);

/* Mirrors ml::InferOptions (src/ml/infer.hpp:38-103), the fields this path implements. A
 * zero-initialised struct past `tta` means: zscore, every tile, no crop, no filter. */
typedef struct fx_infer_opts {
    int patch;      /* tile side P, divisible by 2^(stages-1) */
    double overlap; /* step = (int64)(P * (1 - overlap)) */
    int channel;    /* softmax channel to emit (surface = 1); ignored with sigmoid */
    int sigmoid;    /* 1-class head -> sigmoid */
    int batch;      /* tiles per forward, <= the net's max batch */
    int tta;        /* octahedral test-time augmentation: <= 1 off, else the first min(tta, 48)
                       symmetries, averaged (src/ml/infer.hpp:393-441); each costs a forward */
    int norm;       /* fx_norm */
    int skip_constant; /* 1: tiles whose input voxels all hold one value are not run, they add nothing
                          to the blend (predict-scroll's rule, src/ml/inference.cpp:1487-1496, 1885-1900) */
    int64_t core_org[3]; /* output crop (InferOptions::core_org / core_ext, src/ml/infer.hpp:69-76):
                            tiles still read the whole input, a tile that does not reach the core is not
                            run, and the outputs cover only [core_org, core_org + core_ext) */
    int64_t core_ext[3]; /* <= 0 along an axis: to the end of the input */
    fx_tile_filter_fn tile_filter; /* NULL: every tile */
    void* tile_filter_user;
    int tile[3]; /* per-axis tile (z, y, x) for nets built by fx_net_create_tiled; all 0: the cube of
                    side `patch`, which then must be divisible by 64 as in the reference
                    (src/ml/infer.hpp:459). The reference tiles cubes only; an anisotropic tile is
                    the layer-stack (wide-ink) workload's 64 x 256 x 256, stepped per axis by
                    (int64)(tile[a] * (1 - overlap)) with a Gaussian of sigma tile[a] / 8 per axis.
                    The tile filter's `patch` argument is then tile[0]. TTA needs a cube. */
    int stacks;  /* >= 2: the volume is `stacks` independent volumes of dz / stacks planes each,
                    stacked along z (a batch of layer stacks): tile starts, Gaussian weights and
                    the normalisation run per stack and no tile crosses a stack boundary, so the
                    result equals predicting each stack alone while every forward fills the
                    batch. Each stack must be at least one tile deep; no output crop, no z-slabs.
                    0 or 1: one volume. No reference counterpart (the reference predicts one
                    volume per call, src/ml/infer.hpp:456). */
    /* Resumable prediction (InferOptions::ckpt_path / ckpt_every / weights_hash / input_hash,
       src/ml/infer.hpp:78-96, 136-344), fx_predict_volume / fx_predict_volume_dev only: when
       ckpt_path is set, a checkpoint written in the reference's FXICKPT3 layout (header: dims,
       patch, overlap, tta, tile_shift 0, total / completed tile counts, the two identity hashes,
       the u16 scale, channel, sigmoid, norm; then the accumulator as u16 = (u16)(acc / scale *
       65535 + 0.5)) that matches this call is loaded and the run continues after its completed
       tiles; every ckpt_every tiles (<= 0: 128) the accumulator is saved there (temp + rename, by
       a background thread, a save skipped while the previous one is writing); on success the file
       is removed. Tiles run in the fixed z-major order. Not with an output crop, stacks or a
       non-cubic tile (FX_UNSUPPORTED). NULL: off. */
    const char* ckpt_path;
    int64_t ckpt_every;
    uint64_t weights_hash; /* identity of the weights / input the checkpoint belongs to (0: none) */
    uint64_t input_hash;
} fx_infer_opts;

typedef struct fx_net fx_net;

/* Last error message of the calling thread ("" when none). */
const char* fx_last_error(void);

/* Number of CUDA devices visible (0 when no driver or GPU). */
int fx_device_count(void);

/* Build a 3D UNet from an .fxweights file (FXWT v1, src/ml/weights.hpp:1-10) on device `device`,
 * for tiles of side `patch` and up to `max_batch` tiles per forward. The architecture, stage
 * count, features and classes are read from the tensor names and shapes:
 *   plain UNet      — encoder.stages.{s}.convs.{i}.conv.*, decoder.transpconvs.{t}.*,
 *                     decoder.stages.{t}.convs.{i}.*, decoder.seg_layers.{t}.*
 *   residual UNet   — nets::ResEncUNet (src/ml/nets/resenc_unet.hpp:159-318):
 *                     {encoder|shared_encoder}.stem.convs.0.*, ...stages.{s}.blocks.{b}.conv1/conv2/
 *                     skip.{i}/squeeze_excitation.*, with the decoder under decoder.* or
 *                     task_decoders.<task>.* (BasicBlockD with AvgPool + 1x1 projection skips, scSE). */
fx_status fx_net_create(const char* fxweights_path, int patch, int max_batch, fx_precision precision, int device,
                        fx_net** out);
/* The same for a tile of tile[0] x tile[1] x tile[2] (z, y, x) voxels. A stage downsamples only the
 * axes its stride-2 conv strides (read from the decoder's transposed-conv kernel shape, e.g.
 * (1, 2, 2) for a y/x-only stage); every level's extent must halve evenly. No reference
 * counterpart: the reference's predict path tiles cubes (src/ml/infer.hpp:39, 459). */
fx_status fx_net_create_tiled(const char* fxweights_path, const int tile[3], int max_batch, fx_precision precision,
                              int device, fx_net** out);
void fx_net_destroy(fx_net* net);
/* Static net shape, like TrtNet's batch()/patch()/classes(). fx_net_patch is 0 for a non-cubic tile;
 * fx_net_tile writes (z, y, x) and the per-stage stride masks (bit 2 z, bit 1 y, bit 0 x; stage 0's
 * is 0) into masks[0..cap) when masks is not NULL, returning the stage count. */
int fx_net_patch(const fx_net* net);
int fx_net_tile(const fx_net* net, int tile[3], int* masks, int cap);
int fx_net_max_batch(const fx_net* net);
int fx_net_classes(const fx_net* net);
int fx_net_features(const fx_net* net, int* out, int cap); /* returns the stage count */

/* fp8 only: record per-tensor activation amax over `n` host u8 patches ([n][P][P][P]) in a
 * 16-bit (f16) calibration forward, and fix every activation scale to running-max(amax) / 448. */
fx_status fx_net_calibrate(fx_net* net, const uint8_t* host_patches, int n);
/* The input normalisation (fx_norm) that fx_net_calibrate, fx_net_calibrate_schedule and
 * fx_net_forward apply to their u8 tiles (default zscore); the predict entry points set their own
 * from fx_infer_opts. A net predicting with pct_minmax or unit255 is calibrated under the same. */
fx_status fx_net_set_norm(fx_net* net, int norm);
/* Per-tensor activation scales after calibration (cap entries); returns the count. One per conv
 * layer, in the order encoder convs (stage-major), transposed convs (finest level first),
 * decoder convs (finest level first): the scale of that layer's input activation. */
int fx_net_act_scales(const fx_net* net, float* out, int cap);
/* fp8 only: install previously calibrated scales (same order and count) instead of calibrating. */
fx_status fx_net_set_act_scales(fx_net* net, const float* scales, int count);
/* Precision schedule of an fp8 net (mixed precision, the per-layer counterpart of the
 * reference's sensitive-layer notes, docs/design/fp8-conv3d-sm120.md:71-103): one entry per conv
 * layer in fx_net_act_scales order, FX_PREC_FP8 for e4m3 operands or the net's 16-bit type
 * (FX_PREC_F16 for fp8 nets) to keep that layer on 16-bit operands. Layers that cannot take e4m3
 * (the first conv, input channels not a multiple of 32) stay 16-bit. Default: every eligible
 * layer e4m3. */
fx_status fx_net_set_layer_precision(fx_net* net, const int* precision, int count);
/* Calibrated precision schedule of an fp8 net from n host patches ([n][P][P][P] u8): calibrates the
 * scales if needed, then measures, against the net's own 16-bit forward of the patches, what e4m3
 * operands in each layer alone cost (Dice of the 0.5-thresholded masks, max |dp|) and save (conv
 * time of both operand types, CUDA events), takes layers greedily by time saved per unit of squared
 * Dice loss while the summed squared losses stay within (1 - min_dice)^2 and no layer alone moves a
 * probability by more than max_abs (<= 0: unbounded), runs the result and gives layers back until it
 * meets both bounds. dice / maxabs (either may be NULL) receive the schedule's agreement with the
 * 16-bit forward. The reference's fp8 notes keep their sensitive layers in 16-bit by hand
 * (docs/design/fp8-conv3d-sm120.md:71-103); this measures the sensitivity instead. */
fx_status fx_net_calibrate_schedule(fx_net* net, const uint8_t* host_patches, int n, double min_dice, double max_abs,
                                    double* dice, double* maxabs);
/* The operand precision each conv layer runs with (fx_precision values, fx_net_act_scales order)
 * and, when flops is non-NULL, its algorithmic FLOPs per tile (2 x MACs); returns the count. */
int fx_net_layer_precision(const fx_net* net, int* precision, double* flops, int cap);
/* The weights-file prefix of conv layer i (fx_net_act_scales order), e.g.
 * "decoder.stages.3.convs.0"; NULL when out of range. Valid while the net lives. */
const char* fx_net_layer_name(const fx_net* net, int i);

/* Forward `nb` device-resident u8 tiles ([nb][P][P][P]) through the net and write the selected
 * class probability ([nb][P][P][P] f32, device). Each tile is z-scored on its own (norm_patch).
 * `stream` is a cudaStream_t (NULL = the net's stream). */
fx_status fx_net_forward(fx_net* net, const uint8_t* dev_tiles, int nb, float* dev_prob, int channel, int sigmoid,
                         void* stream);

/* Sliding-window prediction over a host-resident dense u8 volume [dz][dy][dx] (ZYX, x fastest).
 * Outputs (either may be NULL): the normalised probability (f32) and its u8 encoding, both with the
 * crop's dims when opts has an output crop (else the input's). */
fx_status fx_predict_volume(fx_net* net, const uint8_t* host_vol, int64_t dz, int64_t dy, int64_t dx,
                            const fx_infer_opts* opts, float* host_prob, uint8_t* host_u8);

/* fx_predict_volume on device buffers: dev_vol [dz][dy][dx] u8 resident on the net's device; the
 * normalised probability map into dev_prob (f32, the output's dims; may be NULL) and/or its u8
 * encoding into dev_u8 (may be NULL; one of the two is required). Runs asynchronously on `stream`
 * (NULL: the net's stream); the accumulator is dev_prob when given, else the net's workspace. A
 * bounded wait that gave up inside the call is reported by the next fx_net_device_status. No
 * reference counterpart: the reference's predict reads and writes host memory. */
fx_status fx_predict_volume_dev(fx_net* net, const uint8_t* dev_vol, int64_t dz, int64_t dy, int64_t dx,
                                const fx_infer_opts* opts, float* dev_prob, uint8_t* dev_u8, void* stream);

/* Device-resident sliding window restricted to the flat tile range [tile_begin, tile_end) of the
 * z-major tile grid over a (full_dz, dy, dx) volume (z-slab sharding, the tile grid of
 * predict-scroll's global mode, src/ml/inference.cpp:1282-1372). dev_slab holds planes
 * [z_origin, z_origin + slab_dz) of the volume and dev_acc ([slab_dz][dy][dx] f32, caller-zeroed)
 * the matching accumulator planes; every tile of the range must lie inside the slab. Only
 * accumulates (Gaussian-weighted sums); fx_accum_finalize normalises. */
fx_status fx_predict_tiles_dev(fx_net* net, const uint8_t* dev_slab, int64_t slab_dz, int64_t dy, int64_t dx,
                               int64_t z_origin, int64_t full_dz, const fx_infer_opts* opts, int64_t tile_begin,
                               int64_t tile_end, float* dev_acc, void* stream);
/* The device status word of the net's kernels: FX_OK, or FX_INTERNAL with the code in the message
 * when a kernel's bounded wait gave up (the kernel then returns early instead of hanging, and its
 * outputs are undefined). Synchronises the net's stream and clears the word; call it after the
 * stream given to fx_predict_tiles_dev is synchronised. fx_predict_volume and fx_net_forward check
 * it themselves. The reference's counterpart is the worker error path (src/ml/infer.hpp:675-808). */
fx_status fx_net_device_status(fx_net* net);
/* Failure-detection self-test: one small conv launch whose MMA warp waits on a barrier that nothing
 * arrives at, with every wait bounded by wait_ns. The launch ends by itself after about wait_ns and
 * *status_out receives the kernel's status word, the code of the first wait that gave up (0x100: the
 * MMA warp's stage wait, 0x300: the epilogue's accumulator wait); the context stays usable. No reference counterpart (the reference has no device code). */
fx_status fx_selftest_wait_timeout(int device, uint64_t wait_ns, uint32_t* status_out);
/* dev_dst[i] += dev_src[i] over n f32 values: folds the band another GPU accumulated for planes
 * this GPU owns into its own accumulator. dev_src may be another GPU's memory (a peer pointer or an
 * IPC mapping): the kernel then reads it over NVLink. 16-byte aligned pointers take the vector path. */
fx_status fx_accum_add(float* dev_dst, const float* dev_src, int64_t n, void* stream);

/* ---- several GPUs, no collective (z-slab sharding) ----
 * The reference runs one replica per GPU on worker threads over one global tile grid
 * (src/ml/inference.cpp:1129-1188, 1402-1586). Here the z-major tile list of the volume's grid is
 * split into contiguous near-equal ranges, one per GPU; shard r reads input planes [z_lo, z_hi)
 * (every plane its tiles touch), accumulates over the same planes and finalises the planes it owns,
 * [own_lo, own_hi) (a partition of [0, dz)). A shard with no tiles has tile_begin == tile_end. */
typedef struct fx_shard {
    int64_t tile_begin, tile_end;
    int64_t z_lo, z_hi;
    int64_t own_lo, own_hi;
} fx_shard;
/* Writes nshards plans to out (when non-NULL); returns nshards, or 0 on bad arguments. */
int fx_shard_plan(int64_t dz, int64_t dy, int64_t dx, int patch, double overlap, int nshards, fx_shard* out);
/* fx_predict_volume over n nets (normally one per device; nets may share a device), one host thread
 * per net: each uploads its
 * input slab, blends its tile range into its own accumulator window, then (after every device has
 * finished) adds the bands its neighbours accumulated for its owned planes, read from their HBM over
 * NVLink by an add kernel (staged with a peer copy where the devices cannot map each other), and
 * finalises and downloads its owned planes. Same outputs as fx_predict_volume. */
fx_status fx_predict_volume_multi(fx_net* const* nets, int n, const uint8_t* host_vol, int64_t dz, int64_t dy,
                                  int64_t dx, const fx_infer_opts* opts, float* host_prob, uint8_t* host_u8);

/* Device buffers another process can map: with one process per GPU, a shard's accumulator window is
 * allocated here and its CUDA IPC handle (64 bytes) handed to the neighbours through the host, which
 * map it (fx_ipc_open) and fold the bands they own with fx_accum_add reading it over NVLink. The
 * buffer's owner frees it only after every mapping of it is closed. */
fx_status fx_ipc_buffer_alloc(int device, uint64_t bytes, void** dev_ptr, void* handle);
fx_status fx_ipc_buffer_free(int device, void* dev_ptr);
fx_status fx_ipc_open(int device, const void* handle, void** dev_ptr);
fx_status fx_ipc_close(int device, void* dev_ptr);

/* Device timing of the tensor-core convolutions: with profiling enabled every conv launch of
 * this net is bracketed by CUDA events on its stream; fx_net_profile_read synchronises them and
 * returns the summed duration (ms), the algorithmic FLOPs (2 x MACs) of those launches, the
 * part of them run with e4m3 operands, the launch count and (when per_launch is non-NULL) up to
 * `cap` per-launch (ms, FLOPs) pairs in launch order, then clears the record. */
fx_status fx_net_profile(fx_net* net, int enable);
fx_status fx_net_profile_read(fx_net* net, double* conv_ms, double* conv_flops, double* fp8_flops,
                              int64_t* conv_launches, double* per_launch, int cap);
/* The same record summed per conv layer (fx_net_layer_precision order): layer_ms[i] = the summed
 * duration of layer i's launches, for up to `cap` layers; also clears the record. Returns the
 * layer count, or -1 on error (fx_last_error). */
int fx_net_profile_read_layers(fx_net* net, double* layer_ms, int cap);
/* The dense tcgen05 tensor rate of `device`, measured with this library's own kernel: one CTA per SM
 * issuing M = 128, N = 256 MMAs back to back on shared-memory-resident operands (kind::f8f6f4 e4m3
 * for FX_PREC_FP8, kind::f16 for bf16 / f16) into TMEM. `runs` launches of about ms_per_run each:
 * *best_tflops = the fastest (the burst rate), *mean_tflops (may be NULL) = their mean; a single long
 * run gives the sustained, power-capped rate. No reference counterpart (the reference measures
 * none). */
fx_status fx_tc_peak(int device, int precision, double ms_per_run, int runs, double* best_tflops, double* mean_tflops);
/* fx_tc_peak for MMAs of n_cols columns (16..256, a multiple of 16): the rate an M = 128 x N = n_cols
 * tcgen05 MMA shape reaches with its operands in shared memory, i.e. the tensor ceiling of a layer
 * whose MMAs have that width. fx_tc_peak is n_cols = 256. No reference counterpart. */
fx_status fx_tc_rate(int device, int precision, int n_cols, double ms_per_run, int runs, double* best_tflops,
                     double* mean_tflops);
/* Kernel launches issued by this library since the process started. */
unsigned long long fx_kernel_launches(void);
/* Device buffer of 16 u64 cycle counters that conv launches add to when the library is built
 * with FX_CONV_TRACE (producer / MMA issuer / epilogue waiting and working time); NULL detaches.
 * Without that build flag the counters are never touched. */
void fx_conv_trace_buffer(void* dev_counters);

/* ---- streaming global accumulator: GlobalAccum (src/ml/global_accum.hpp:37-198) on the device ----
 * The global tile grid of predict-scroll over the 64-aligned bbox [org, org + ext): tile_starts
 * of `patch` / `overlap` along each axis of ext. The f32 accumulator is a window of
 * window_planes planes in HBM (rounded up to 64; 0 = patch + 64, enough for a z-sweep that
 * finalizes the chunk rows below each tile row before running it), starting at the finalize floor.
 * Chunk rows are 64 planes. Calls on one accumulator are serialised by the caller. */
typedef struct fx_gaccum fx_gaccum;
fx_status fx_gaccum_create(const int64_t* org3, const int64_t* ext3, int patch, double overlap, int64_t window_planes,
                           int device, fx_gaccum** out);
void fx_gaccum_destroy(fx_gaccum* acc);
int64_t fx_gaccum_chunk_rows(const fx_gaccum* acc);    /* ceil(ext.z / 64) */
int64_t fx_gaccum_floor_row(const fx_gaccum* acc);     /* chunk rows below are finalized */
int64_t fx_gaccum_window_planes(const fx_gaccum* acc);
int64_t fx_gaccum_tile_rows(const fx_gaccum* acc);     /* tile rows (z starts) of the grid */
int64_t fx_gaccum_row_start(const fx_gaccum* acc, int64_t zi); /* bbox-local z start of tile row zi */
/* Resume: chunk rows below floor_row are already finalized; contributions below are dropped
 * (GlobalAccum::set_floor_row). */
fx_status fx_gaccum_set_floor_row(fx_gaccum* acc, int64_t floor_row);
/* Gaussian-blend one host P^3 probability tile at scroll coordinates (GlobalAccum::scatter).
 * Fails with FX_INVALID_ARGUMENT when the tile reaches past the window. */
fx_status fx_gaccum_scatter(fx_gaccum* acc, int64_t z0, int64_t y0, int64_t x0, const float* host_prob);
/* Run every tile of tile row zi through `net` and blend it in: host_planes holds bbox-local
 * planes [row_start(zi), min(row_start(zi) + patch, ext.z)) of the u8 input, [n][ext.y][ext.x]. */
fx_status fx_gaccum_predict_row(fx_gaccum* acc, fx_net* net, int64_t zi, const uint8_t* host_planes,
                                const fx_infer_opts* opts);
/* Finalize chunk rows [floor_row, row_lim) (GlobalAccum::finalize_rows_below): normalise by
 * Wz.Wy.Wx, (u8)(clamp(v, 0, 1) * 255 + 0.5), written to host_u8 as the planes
 * [floor_row * 64, min(row_lim * 64, ext.z)) x ext.y x ext.x (cap_bytes >= that); *planes_out
 * receives their count. The window then starts at row_lim. */
fx_status fx_gaccum_finalize_below(fx_gaccum* acc, int64_t row_lim, uint8_t* host_u8, int64_t cap_bytes,
                                   int64_t* planes_out);
/* Composing the accumulators of several GPUs that each run a contiguous range of tile rows (the
 * out-of-core run over N GPUs; the reference shares one host GlobalAccum between its device
 * threads, src/ml/inference.cpp:1402-1586). The chunk rows a range's first rows share with the
 * range below are finished by the owner below: the upper accumulator copies those planes out
 * (fx_gaccum_export_planes, bbox-local planes [z0, z0 + n) of its window into dev_dst, f32 on its
 * device) and drops them from its window without finalizing (fx_gaccum_discard_below); the owner
 * adds them into its own window (fx_gaccum_add_planes: dev_src may be a peer's or IPC-mapped
 * memory, read by a kernel on the owner's device) before finalizing them. No reference
 * counterpart as functions: they split GlobalAccum's shared state across devices. */
fx_status fx_gaccum_export_planes(fx_gaccum* acc, int64_t z0, int64_t n, float* dev_dst);
fx_status fx_gaccum_add_planes(fx_gaccum* acc, int64_t z0, int64_t n, const float* dev_src);
fx_status fx_gaccum_discard_below(fx_gaccum* acc, int64_t row_lim);

/* ---- tiling math (host) ---- */
/* Start positions along one axis; returns the count (writes at most cap). */
int64_t fx_tile_starts(int64_t dim, int patch, double overlap, int64_t* out, int64_t cap);
void fx_gaussian1d(int n, float* out);
/* Accumulated Gaussian weight over [c0, c0+cn) of an axis of length dim. */
void fx_weight_profile(const float* g, int patch, const int64_t* starts, int64_t nstarts, int64_t c0, int64_t cn,
                       int64_t dim, float* out);

/* ---- device kernels, for parity tests and custom drivers (device pointers) ---- */
/* z-score `ntiles` tiles at the given origins of a device u8 volume into f32 [ntiles][P^3]. */
fx_status fx_norm_tiles(const uint8_t* dev_vol, int64_t dz, int64_t dy, int64_t dx, const int64_t* host_origins,
                        int ntiles, int patch, float* dev_out, void* stream);
/* fx_norm_tiles with any of the reference's patch normalisations (fx_norm: zscore, pct_minmax,
 * unit255; src/ml/infer.hpp:107-134, 350-385): the dense u8 filler + detail::norm_patch. */
fx_status fx_norm_tiles_mode(const uint8_t* dev_vol, int64_t dz, int64_t dy, int64_t dx, const int64_t* host_origins,
                             int ntiles, int patch, int norm, float* dev_out, void* stream);
/* fx_norm_tiles without any device allocation. No reference counterpart: the reference
 * allocates its patch buffers per call. This one keeps its scratch (tile origins and the
 * per-tile exact sums) in a static 160 KiB __device__ array, so it serves callers that must not
 * allocate: a process that has committed the device's memory to its volume and accumulators,
 * and callers with work in flight on other streams, which cudaFree's implicit device-wide
 * synchronisation would stall. Limit: ntiles <= 4096 per call; more is rejected with
 * FX_INVALID_ARGUMENT. The first call on each device resolves the scratch's address
 * (cudaGetSymbolAddress) and should come before any stream capture. Calls that overlap in time
 * on the same device share the scratch and race. Synchronises `stream` before returning. */
fx_status fx_norm_tiles_noalloc(const uint8_t* dev_vol, int64_t dz, int64_t dy, int64_t dx,
                                const int64_t* host_origins, int ntiles, int patch, float* dev_out, void* stream);
/* One 3x3x3 conv (pad 1, stride 1 or 2, no bias) in f32 NCDHW device tensors, computed by the
 * tcgen05 kernel with `precision` operands (fp8: per-output-channel weight scales and a per-tensor
 * input scale), f32 accumulate, the output rounded once to f16 as the net's pre-norm store does.
 * Also writes per-channel mean and biased variance of the f32 output per batch item into
 * dev_stats [B][Cout][2] when non-NULL. */
fx_status fx_conv3d(const float* dev_x, int B, int Cin, int D, int H, int W, const float* dev_w, int Cout,
                    int stride, fx_precision precision, float* dev_y, float* dev_stats, void* stream);
/* nn::ConvTranspose3d(k=2, s=2) with bias, f32 NCDHW device tensors, `precision` operands,
 * output rounded once to f16. */
fx_status fx_conv_transpose2(const float* dev_x, int B, int Cin, int D, int H, int W, const float* dev_w,
                             const float* dev_bias, int Cout, fx_precision precision, float* dev_y, void* stream);
/* Normalise planes [z_begin, z_end) of an f32 accumulator [dz][dy][dx] by the factorised weights
 * Wz[z] Wy[y] Wx[x] and encode u8; dev_prob / dev_u8 (either may be NULL) receive just those
 * planes, plane z_begin first. */
fx_status fx_accum_finalize(const float* dev_acc, int64_t dz, int64_t dy, int64_t dx, int64_t z_begin, int64_t z_end,
                            const float* dev_wz, const float* dev_wy, const float* dev_wx, float* dev_prob,
                            uint8_t* dev_u8, void* stream);

/* ---- .fxvol archives and the chunk codec ---------------------------------------------------
 * A 64^3 chunk is one tile of 4^3 DCT-16 blocks whose magnitude categories share up to 8 clustered
 * rANS tables. Payloads and files are bit-compatible with the reference's codec and container. */
typedef struct fx_fxvol fx_fxvol;

typedef struct fx_fxvol_info {
    int64_t dims[3];  /* LOD-0 z, y, x */
    float q, hf_exp, dz_frac;
    uint32_t nlods;
    int32_t src_dtype; /* codec::DType: 0 u8, 1 u16, 2 u32, 3 s8, 4 s16, 5 s32, 6 f16, 7 f32 */
    int32_t sealed;    /* a finalize()d (SEALED) archive */
} fx_fxvol_info;

/* VolumeArchive::open, read-only (archive.hpp:161-262). */
fx_status fx_fxvol_open(const char* path, fx_fxvol** out);
/* VolumeArchive::create (archive.hpp:135-158): DctParams{.q = q}, hf_exp 0.65, dz_frac 0.80. */
fx_status fx_fxvol_create(const char* path, int64_t dz, int64_t dy, int64_t dx, float q, int32_t src_dtype,
                          fx_fxvol** out);
/* dims() / params() / nlods() / src_dtype() */
fx_status fx_fxvol_get_info(const fx_fxvol* a, fx_fxvol_info* out);
/* coverage() (0 ABSENT, 1 ZERO, 2 REAL) and, for REAL chunks, the crc-checked payload, valid until
 * fx_fxvol_close (archive.hpp:376-399 up to the decode). */
fx_status fx_fxvol_chunk_payload(const fx_fxvol* a, int lod, int64_t cz, int64_t cy, int64_t cx, int* coverage,
                                 const uint8_t** payload, uint64_t* len);
/* write_chunk_payload (archive.hpp:350-362); len 0 records a ZERO chunk (commit_encoded_). */
fx_status fx_fxvol_write_chunk_payload(fx_fxvol* a, int lod, int64_t cz, int64_t cy, int64_t cx,
                                       const uint8_t* payload, uint64_t len);
/* the LOD count written at close (write_volume sets it after the pyramid, archive.hpp:428-439) */
fx_status fx_fxvol_set_nlods(fx_fxvol* a, uint32_t nlods);
/* close(): commit + trim for writers (archive.hpp:867-894); frees the handle. */
fx_status fx_fxvol_close(fx_fxvol* a);
/* read_volume_as<u8>(0) (archive.hpp:550-590), decoded on `device`: out holds dims z*y*x voxels. */
fx_status fx_fxvol_read_volume_u8(const fx_fxvol* a, int device, uint8_t* out);
/* write_volume<u8> (archive.hpp:418-440): LOD 0 and the 2x octave pyramid, encoded on `device`. */
fx_status fx_fxvol_write_volume_u8(fx_fxvol* a, const uint8_t* vol, int device);
/* decode_tile_dct over n payloads (payloads + offsets[k], lengths[k] bytes) into n 64^3 tiles:
 * u8 (out_u8) and/or the f32 reconstruction (out_f32); either may be NULL, not both. */
fx_status fx_fxvol_decode_tiles(const uint8_t* payloads, uint64_t payload_bytes, const uint64_t* offsets,
                                const uint32_t* lengths, int64_t n, float q, float hf_exp, float dz_frac, int device,
                                uint8_t* out_u8, float* out_f32);
/* encode_tile_dct over n 64^3 tiles (u8 or f32, exactly one non-NULL) into out (cap bytes):
 * payload k at out + offsets[k], lengths[k] bytes. FX_INVALID_ARGUMENT if cap is too small. */
fx_status fx_fxvol_encode_tiles(const uint8_t* tiles_u8, const float* tiles_f32, int64_t n, float q, float hf_exp,
                                float dz_frac, int device, uint8_t* out, uint64_t cap, uint64_t* offsets,
                                uint32_t* lengths);
/* predict-surface over archives: decode the u8 input archive's LOD 0 on the net's device, predict
 * (opts as fx_predict_volume), write the u8 prediction as an .fxvol at q = out_q (<= 0: 32) with
 * its LOD pyramid. The volume stays on the device from decode to encode. */
fx_status fx_predict_fxvol(fx_net* net, const char* in_path, const char* out_path, const fx_infer_opts* opts,
                           float out_q);

#ifdef __cplusplus
}
#endif

#endif /* FENIX_B200_H */
