/* fxo.h — CPU oracle for the surface-prediction inference path. TEST INFRASTRUCTURE ONLY:
 * it is the checker the GPU path is compared against (tests/, the smoke check and the bench's
 * CPU-baseline leg); nothing in the product calls it.
 *
 * A plain-C restatement (fp32 activations, double statistics, OpenMP) of the reference's
 * algorithm, each function citing the reference file:line it follows:
 *   tiling          src/ml/tiling.hpp:16-42, src/ml/infer.hpp:499-509, src/ml/global_accum.hpp:29-35
 *   patch fill      src/ml/inference.cpp:309-321 (dense u8 filler, core/volume.hpp at_clamped)
 *   normalisation   src/ml/infer.hpp:350-385 (norm_patch, zscore)
 *   net             src/ml/nets/resenc_unet.hpp:35-52 (ConvNormAct), 141-158 (ConvStack),
 *                   197-239 (Decoder: ConvTranspose3d(2, s2) -> cat(up, skip) -> convs -> 1x1 head)
 *   head            src/ml/infer.hpp:760-767 (softmax channel select / sigmoid, nan_to_num)
 *   blend           src/ml/infer.hpp:631-653 (scatter), 510-521 (normalize)
 *   u8 encode       src/ml/inference.cpp:343-351
 * The conv/InstanceNorm/transposed-conv arithmetic itself lives in libtorch (ATen) in the
 * reference; it is restated here from its published definitions (PyTorch 2.11 semantics:
 * zero padding, biased variance, eps inside the square root).
 */
#ifndef FXO_H
#define FXO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

int64_t fxo_tile_starts(int64_t dim, int patch, double overlap, int64_t* out, int64_t cap);
void fxo_gaussian1d(int n, float* out);
void fxo_weight_profile(const float* g, int patch, const int64_t* starts, int64_t nstarts, int64_t c0, int64_t cn,
                        int64_t dim, float* out);

void fxo_fill_patch_u8(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, int64_t z0, int64_t y0, int64_t x0,
                       int P, float* out);
void fxo_norm_patch_zscore(float* x, int P);
/* the same over a tz x ty x tx tile */
void fxo_fill_tile_u8(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, int64_t z0, int64_t y0, int64_t x0,
                      int tz, int ty, int tx, float* out);
void fxo_norm_tile_zscore(float* x, int tz, int ty, int tx);

void fxo_conv3d(const float* x, int B, int Cin, int D, int H, int W, const float* w, const float* bias, int Cout,
                int stride, float* y);
/* stride (sz, sy, sx), each 1 or 2 */
void fxo_conv3d_s(const float* x, int B, int Cin, int D, int H, int W, const float* w, const float* bias, int Cout,
                  int sz, int sy, int sx, float* y);
void fxo_instance_norm_act(float* x, int B, int C, int64_t S, const float* gamma, const float* beta, float eps,
                           int act, float slope);
void fxo_conv_transpose2(const float* x, int B, int Cin, int D, int H, int W, const float* w, const float* bias,
                         int Cout, float* y);
/* kernel = stride = (kz, ky, kx), each 1 or 2; weights [Cin][Cout][kz][ky][kx] */
void fxo_conv_transpose_s(const float* x, int B, int Cin, int D, int H, int W, const float* w, const float* bias,
                          int Cout, int kz, int ky, int kx, float* y);
void fxo_head(const float* x, int B, int C, int64_t S, const float* w, const float* b, int ncls, int channel,
              int sigmoid, float* prob);

typedef struct fxo_net fxo_net;
/* Plain UNet from an .fxweights file (names as in include/fenix_b200.h). NULL on error. A stage's
 * stride (z, y, x) is the kernel shape of the transposed conv that undoes it (2 x 2 x 2 for the
 * surface nets, 1 x 2 x 2 for a y/x-only stage). */
fxo_net* fxo_net_load(const char* path);
void fxo_net_free(fxo_net* net);
int fxo_net_stages(const fxo_net* net);
/* 1 when a tz x ty x tx tile halves evenly through every stage's strides */
int fxo_net_tile_ok(const fxo_net* net, int tz, int ty, int tx);
/* x: [B][P^3] normalised input; prob: [B][P^3] selected-class probability. */
int fxo_net_forward(const fxo_net* net, const float* x, int B, int P, int channel, int sigmoid, float* prob);
int fxo_net_forward_tiled(const fxo_net* net, const float* x, int B, int tz, int ty, int tx, int channel,
                          int sigmoid, float* prob);

/* predict_surface_filled over a dense u8 volume: tiles, norm, forward, blend, normalise. */
int fxo_predict_surface(const fxo_net* net, const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, int P,
                        double overlap, int channel, int sigmoid, float* prob);
/* the same with a tz x ty x tx tile (per-axis starts, Gaussians of sigma t / 8 and weight profiles) */
int fxo_predict_tiled(const fxo_net* net, const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, int tz, int ty,
                      int tx, double overlap, int channel, int sigmoid, float* prob);
void fxo_prob_to_u8(const float* p, int64_t n, uint8_t* out);

#ifdef __cplusplus
}
#endif

#endif
