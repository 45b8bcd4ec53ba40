// fxvol.cuh — the .fxvol chunk codec on the device: a 64^3 tile is 4^3 DCT-16 blocks whose
// magnitude categories share up to 8 clustered rANS tables (src/codec/dct_block.hpp:318-588).
//
// Decode (fxv_dec_*): a parse kernel (one thread per tile: DC / nsig varints, context map, plane
// headers), a rANS kernel (one warp per category plane, slot table in shared memory), a context walk
// (one thread per tile — the clustered streams and the raw bit stream are consumed in coefficient
// order, so a tile is inherently serial), and a reconstruction kernel (one CTA per tile: inverse
// DCT-16 of every block through shared memory, the quant-gated deblock in the reference's order,
// u8 rounding and the scatter into the destination volume).
// Encode (fxv_enc_*): quantisation (one CTA per block: gather with edge replication, DC, forward
// DCT-16, dead-zone quantiser), context histograms (one CTA per block), context clustering (one
// warp per tile), RDOQ and symbol emission (one thread per block), rANS (one thread per plane) and
// payload assembly (one warp per tile).
// All float arithmetic uses round-to-nearest intrinsics without contraction, in the order of the
// CPU restatement, so device and CPU payloads and reconstructions agree bit for bit.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

namespace fxk {

// DctParams (src/codec/dct_block.hpp:26-37) plus the tables the host derives from them: the
// per-frequency-sum step (dct_block.hpp:91-94, powf) and the DCT-16 half bases (dct.hpp:36-53).
struct FxvParams {
    float q = 32.f, hf_exp = 0.65f, dz_frac = 0.80f, rdoq_lambda = 0.15f, deblock_beta = 2.5f, deblock_tc = 0.5f;
    int rdoq = 1, deblock = 1, dc_predict = 1;
    float stepv[48];
    float me[8][8], mo[8][8];
};
FxvParams fxv_make_params(float q, float hf_exp = 0.65f, float dz_frac = 0.80f);

// One tile to decode: its payload span in the blob and its voxel origin in the destination.
struct FxvDecTile {
    uint64_t off;
    uint32_t len;
    uint32_t pad;
    int64_t z0, y0, x0;
};

// One tile to encode: its voxel origin in the source (edge-replicated at the volume's far faces).
struct FxvEncTile {
    int64_t z0, y0, x0;
};

}  // namespace fxk

namespace fxh {

struct CodecStatus {
    int code = 0;  // 0 ok, 5 decode error (corrupt payload), 8 internal
    std::string msg;
};

// Device codec with its scratch (grown on demand, kept for the object's lifetime). All calls are
// stream-ordered on `s`; results are complete when the call returns.
class FxvCodec {
  public:
    FxvCodec() = default;
    FxvCodec(const FxvCodec&) = delete;
    FxvCodec& operator=(const FxvCodec&) = delete;
    ~FxvCodec();

    // Decode n tiles whose payloads sit in device memory at d_blob. u8 voxels go to d_out
    // (dims dz, dy, dx; voxels outside it are dropped); with d_recon, tile k's f32 reconstruction
    // (after deblocking, before rounding) also goes to d_recon + k * 64^3.
    CodecStatus decode(const uint8_t* d_blob, const fxk::FxvDecTile* tiles, int64_t n, const fxk::FxvParams& p,
                       uint8_t* d_out, int64_t dz, int64_t dy, int64_t dx, float* d_recon, cudaStream_t s);

    // Encode n tiles of a u8 (src8) or f32 (src32) device volume. Appends the payloads to `payload`
    // and one (offset, length) per tile. With zero_slots, a tile whose voxels are all zero gets
    // length 0 (the archive's ZERO slot, archive.hpp:321-338); without, every tile is encoded
    // (encode_tile_dct).
    CodecStatus encode(const uint8_t* src8, const float* src32, int64_t dz, int64_t dy, int64_t dx,
                       const fxk::FxvEncTile* tiles, int64_t n, const fxk::FxvParams& p, std::vector<uint8_t>& payload,
                       std::vector<uint64_t>& offsets, std::vector<uint32_t>& lengths, cudaStream_t s,
                       bool zero_slots);

    // Device kernel launches of the last call (for the launch-count claim of the bench).
    int64_t launches() const { return launches_; }

  private:
    void* grow(void*& p, size_t& cap, size_t want);
    CodecStatus tables(cudaStream_t s);
    int dev_ = -1;
    void* scan_ = nullptr;  // ScanE[4096], then the rank table u16[4096]
    void *hdr_ = nullptr, *syms_ = nullptr, *ent_ = nullptr, *recon_ = nullptr, *ctr_ = nullptr;
    size_t hdr_cap_ = 0, syms_cap_ = 0, ent_cap_ = 0, recon_cap_ = 0, ctr_cap_ = 0;
    void *elev_ = nullptr, *ecoef_ = nullptr, *eblk_ = nullptr, *ehdr_ = nullptr, *ework_ = nullptr, *eout_ = nullptr,
         *eres_ = nullptr;
    size_t elev_cap_ = 0, ecoef_cap_ = 0, eblk_cap_ = 0, ehdr_cap_ = 0, ework_cap_ = 0, eout_cap_ = 0, eres_cap_ = 0;
    void* htiles_ = nullptr;
    size_t htiles_cap_ = 0;
    void* pinned_ = nullptr;
    size_t pinned_cap_ = 0;
    int64_t launches_ = 0;
};

}  // namespace fxh
