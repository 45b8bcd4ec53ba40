/* fxv.h — CPU oracle for the .fxvol chunk codec (64^3 tile = 4^3 DCT-16 blocks sharing clustered
 * rANS tables). TEST INFRASTRUCTURE ONLY: the checker the device codec is compared against (tests/,
 * the bench's CPU-baseline leg); nothing in the product calls it.
 *
 * A plain-C restatement of the reference's tile codec, each part citing the reference file:line:
 *   DCT-16          src/codec/dct.hpp:27-94 (orthonormal DCT-II / DCT-III, even/odd half bases)
 *   rANS            src/codec/rans.hpp:22-279 (12-bit model, 1 or 4 interleaved states)
 *   planes, bits    src/codec/entropy.hpp:61-207 (LEB128 varints, sparse freq tables, LSB-first bits)
 *   tile encode     src/codec/dct_block.hpp:318-484 (DC/nsig causal prediction, dead-zone quant,
 *                   band x neighbour-sum contexts, greedy context clustering, RDOQ, end-of-block)
 *   tile decode     src/codec/dct_block.hpp:492-588 (+ quant-gated deblock, dct_block.hpp:267-309)
 * Arithmetic order is fixed (f32 multiply-then-add, no contraction; 3D transform passes along x, y,
 * then z) and is the one the device kernels use, so the two agree bit for bit. The cost model's
 * log2 is glibc's (mode 0, as the reference) or a portable series both sides evaluate identically
 * (mode 1, the device's): log2 x = e + 2 atanh((m-1)/(m+1)) / ln 2, m in [sqrt(1/2), sqrt(2)).
 *
 * Parity: pinned to the reference's own dct_block.hpp / entropy.hpp / rans.hpp compiled here
 * (oracle/ref_fxvol.cpp), whose Clang-only DCT header is replaced by a scalar DCT-16 of the same
 * basis (oracle/shim_codec/codec/dct.hpp).
 */
#ifndef FXV_H
#define FXV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* DctParams (src/codec/dct_block.hpp:26-37) */
typedef struct fxv_params {
    float q, hf_exp, dz_frac;
    int rdoq;
    float rdoq_lambda;
    int deblock;
    float deblock_beta, deblock_tc;
    int dc_predict;
} fxv_params;

void fxv_params_default(fxv_params* p, float q);

/* 16^3 block transforms in place (z, y, x order, x fastest) */
void fxv_dct3_fwd(float* blk);
void fxv_dct3_inv(float* blk);

/* Decode one 64^3 tile payload. recon (f32, after deblocking) and/or out_u8 may be NULL.
 * Returns 0, or a negative error code (the reference's decode_error cases). */
int fxv_decode_tile(const uint8_t* payload, size_t len, const fxv_params* p, float* recon, uint8_t* out_u8);

/* Encode one 64^3 tile (u8 or f32 source). Returns the payload length, or -1 if cap is too small.
 * log2_mode: 0 glibc log2, 1 the portable series. */
int64_t fxv_encode_tile_u8(const uint8_t* tile, const fxv_params* p, int log2_mode, uint8_t* out, size_t cap);
int64_t fxv_encode_tile_f32(const float* tile, const fxv_params* p, int log2_mode, uint8_t* out, size_t cap);

/* The portable log2 (mode 1), exposed for tests. */
double fxv_log2_series(double x);

/* rANS byte-plane coder (entropy.hpp encode_plane / decode_plane), exposed for tests.
 * encode returns the bytes written (or -1 if cap is too small); decode returns the plane length
 * (or a negative error) and advances *pos. */
int64_t fxv_encode_plane(const uint8_t* plane, size_t n, uint8_t* out, size_t cap);
int64_t fxv_decode_plane(const uint8_t* in, size_t len, size_t* pos, uint32_t max_n, uint8_t* out);

/* crc32c (archive.hpp:47-59) and the chunk Morton key (archive.hpp:61-74) */
uint32_t fxv_crc32c(const uint8_t* p, size_t n);
uint64_t fxv_morton3(uint64_t z, uint64_t y, uint64_t x);

#ifdef __cplusplus
}
#endif

#endif
