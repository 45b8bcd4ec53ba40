// fxvol_archive.hpp — the .fxvol v5 container on the host (src/codec/archive.hpp): two crc32c
// superblock slots, one 3-level (12+12+12 bit) compressed-Morton radix page table per LOD, and
// blobs of [payload][u32 crc32c]. The writer keeps the file image in memory and allocates nodes and
// blobs in the reference's order (root, level-1 node, leaf, blob per chunk, 8-byte aligned bump
// allocation, leaves initialised to the ABSENT sentinel), so the same payloads written in the same
// order give a byte-identical file. The reader maps the file read-only and validates every offset
// the way archive.hpp does before following it.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace fxh {

struct FxvolMeta {
    int64_t dims[3] = {0, 0, 0};
    float q = 8.f, hf_exp = 0.65f, dz_frac = 0.80f;
    uint32_t nlods = 1;
    uint32_t dtype = 0;  // codec::DType (0 = u8)
    uint64_t data_off = 0;
};

enum FxvolCoverage { kAbsent = 0, kZero = 1, kReal = 2 };

uint32_t crc32c(const uint8_t* p, size_t n);
uint64_t morton3(uint64_t z, uint64_t y, uint64_t x);
uint32_t plan_nlods(const int64_t dims[3]);  // octaves down to one 64^3 chunk (archive.hpp:905-912)
void dims_at(const int64_t dims[3], int lod, int64_t out[3]);

class FxvolArchive {
  public:
    ~FxvolArchive();
    // VolumeArchive::open (read-only). Returns an empty string or the error message.
    std::string open(const std::string& path);
    // VolumeArchive::create: an empty archive (superblock slot A, commit 1) in memory.
    std::string create(const std::string& path, const int64_t dims[3], float q, float hf_exp, float dz_frac,
                       uint32_t dtype);
    const FxvolMeta& meta() const { return m_; }
    bool writable() const { return writable_; }
    // Coverage and, for REAL chunks, the payload (crc-checked; valid until close).
    std::string chunk(int lod, int64_t cz, int64_t cy, int64_t cx, int* coverage, const uint8_t** payload,
                      uint64_t* len) const;
    // commit_encoded_ / write_chunk_payload: len 0 records a ZERO slot.
    std::string put(int lod, int64_t cz, int64_t cy, int64_t cx, const uint8_t* payload, uint64_t len);
    void set_nlods(uint32_t n) { m_.nlods = n; }
    // commit + close: superblock slot B (commit 2), file trimmed to the committed end.
    std::string close();

  private:
    uint64_t alloc(uint64_t n, bool zero);
    void superblock(uint64_t seq);
    bool in_bounds(uint64_t off, uint64_t need, uint64_t hz) const { return off <= hz && need <= hz - off; }
    uint64_t rd64(uint64_t off) const;
    std::string path_;
    FxvolMeta m_;
    uint64_t roots_[20] = {};
    bool writable_ = false;
    // writer image
    std::vector<uint8_t> img_;
    uint64_t cursor_ = 0, committed_ = 0;
    // reader mapping
    const uint8_t* map_ = nullptr;
    uint64_t map_len_ = 0, hz_ = 0;
    int fd_ = -1;
};

}  // namespace fxh
