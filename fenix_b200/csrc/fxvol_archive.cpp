// fxvol_archive.cpp — see fxvol_archive.hpp. Layout constants and checks follow
// src/codec/archive.hpp:42-130 (superblock fields, radix geometry), 161-262 (open), 317-360
// (chunk writes), 376-399 (chunk reads), 867-894 (commit, close), 1067-1151 (radix walk,
// allocation, superblock write).
#include "fxvol_archive.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>

namespace fxh {

namespace {
constexpr uint32_t kMagic = 0x4c565846u;  // "FXVL"
constexpr uint32_t kVersion = 5;
constexpr uint64_t kNodeEnt = 4096, kSuper = 4096, kDataStart = 2 * kSuper, kMaxLod = 20;
constexpr uint64_t kLodRootOff = 68, kDataOffField = kLodRootOff + 8 * kMaxLod, kSbCrcLen = kDataOffField + 8;
constexpr uint64_t kAbsentOff = ~0ull;  // slot offset sentinel: ABSENT
constexpr uint64_t kNodeBytes = kNodeEnt * 8, kLeafBytes = kNodeEnt * 16;
constexpr int64_t kMaxAxis = 1ll << 18;

template <class T>
T ld(const uint8_t* p) {
    T v;
    std::memcpy(&v, p, sizeof v);
    return v;
}
template <class T>
void st(uint8_t* p, T v) {
    std::memcpy(p, &v, sizeof v);
}
uint64_t part1by2(uint64_t x) {
    x &= 0x1fffffull;
    x = (x | (x << 32)) & 0x1f00000000ffffull;
    x = (x | (x << 16)) & 0x1f0000ff0000ffull;
    x = (x | (x << 8)) & 0x100f00f00f00f00full;
    x = (x | (x << 4)) & 0x10c30c30c30c30c3ull;
    x = (x | (x << 2)) & 0x1249249249249249ull;
    return x;
}
bool fits_one(const int64_t d[3]) { return d[0] <= 64 && d[1] <= 64 && d[2] <= 64; }
}  // namespace

uint32_t crc32c(const uint8_t* p, size_t n) {
    static const auto table = [] {
        std::vector<uint32_t> t(256);
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ 0x82f63b78u : c >> 1;
            t[i] = c;
        }
        return t;
    }();
    uint32_t crc = ~0u;
    for (size_t i = 0; i < n; ++i) crc = table[(crc ^ p[i]) & 0xffu] ^ (crc >> 8);
    return ~crc;
}

uint64_t morton3(uint64_t z, uint64_t y, uint64_t x) { return (part1by2(z) << 2) | (part1by2(y) << 1) | part1by2(x); }

void dims_at(const int64_t dims[3], int lod, int64_t out[3]) {
    int64_t d[3] = {dims[0], dims[1], dims[2]};
    for (int i = 0; i < lod; ++i)
        for (int a = 0; a < 3; ++a) d[a] = (d[a] + 1) / 2;
    for (int a = 0; a < 3; ++a) out[a] = d[a];
}

uint32_t plan_nlods(const int64_t dims[3]) {
    int64_t d[3] = {dims[0], dims[1], dims[2]};
    uint32_t n = 1;
    while (!fits_one(d) && n < kMaxLod) {
        for (int a = 0; a < 3; ++a) d[a] = (d[a] + 1) / 2;
        ++n;
    }
    return n;
}

FxvolArchive::~FxvolArchive() {
    if (map_) munmap(const_cast<uint8_t*>(map_), map_len_);
    if (fd_ >= 0) ::close(fd_);
}

uint64_t FxvolArchive::rd64(uint64_t off) const {
    return writable_ ? ld<uint64_t>(img_.data() + off) : ld<uint64_t>(map_ + off);
}

std::string FxvolArchive::open(const std::string& path) {
    path_ = path;
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) return "cannot open " + path;
    struct stat sb {};
    if (fstat(fd_, &sb) != 0) return "cannot stat " + path;
    map_len_ = static_cast<uint64_t>(sb.st_size);
    if (map_len_ < kDataStart) return "truncated .fxvol";
    void* p = mmap(nullptr, map_len_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (p == MAP_FAILED) return "mmap failed";
    map_ = static_cast<const uint8_t*>(p);
    int best = -1;
    uint64_t best_seq = 0;
    for (int s = 0; s < 2; ++s) {
        const uint8_t* b = map_ + s * kSuper;
        if (ld<uint32_t>(b) != kMagic || ld<uint32_t>(b + 4) != kVersion) continue;
        if (crc32c(b, kSbCrcLen) != ld<uint32_t>(b + kSbCrcLen)) continue;
        const uint64_t seq = ld<uint64_t>(b + 8);
        if (best < 0 || seq > best_seq) {
            best = s;
            best_seq = seq;
        }
    }
    if (best < 0) return "no valid superblock";
    const uint8_t* b = map_ + best * kSuper;
    const uint64_t eof = ld<uint64_t>(b + 16);
    m_.nlods = ld<uint32_t>(b + 24);
    const uint32_t dt = ld<uint32_t>(b + 28);
    if ((dt & 0xff) > 7) return "bad src dtype";
    m_.dtype = dt & 0xff;
    for (int a = 0; a < 3; ++a) m_.dims[a] = ld<int64_t>(b + 32 + 8 * a);
    m_.q = ld<float>(b + 56);
    m_.hf_exp = ld<float>(b + 60);
    m_.dz_frac = ld<float>(b + 64);
    if (m_.nlods < 1 || m_.nlods > kMaxLod) return "bad nlods";
    for (int a = 0; a < 3; ++a)
        if (m_.dims[a] <= 0 || m_.dims[a] > kMaxAxis) return "dims out of range";
    if (!(m_.q > 0.0f) || !std::isfinite(m_.q)) return "bad quant step";
    for (uint64_t l = 0; l < kMaxLod; ++l) roots_[l] = ld<uint64_t>(b + kLodRootOff + 8 * l);
    m_.data_off = ld<uint64_t>(b + kDataOffField);
    if (eof > map_len_ || eof < kDataStart) return "corrupt eof";
    hz_ = eof;
    for (uint32_t l = 0; l < m_.nlods; ++l)
        if (roots_[l] != 0 && !in_bounds(roots_[l], kNodeBytes, hz_)) return "corrupt root";
    return {};
}

std::string FxvolArchive::create(const std::string& path, const int64_t dims[3], float q, float hf_exp, float dz_frac,
                                 uint32_t dtype) {
    for (int a = 0; a < 3; ++a)
        if (dims[a] <= 0 || dims[a] > kMaxAxis) return "dims out of range";
    if (!(q > 0.0f) || !std::isfinite(q)) return "bad quant step";
    if (dtype > 7) return "bad src dtype";
    path_ = path;
    for (int a = 0; a < 3; ++a) m_.dims[a] = dims[a];
    m_.q = q;
    m_.hf_exp = hf_exp;
    m_.dz_frac = dz_frac;
    m_.dtype = dtype;
    m_.nlods = plan_nlods(dims);
    writable_ = true;
    img_.assign(kDataStart, 0);
    cursor_ = committed_ = kDataStart;
    superblock(1);
    // the file exists from create on (archive.hpp:145-156); close() writes the final image
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) return "cannot create " + path;
    const bool ok = std::fwrite(img_.data(), 1, img_.size(), f) == img_.size();
    std::fclose(f);
    return ok ? std::string() : "cannot write " + path;
}

uint64_t FxvolArchive::alloc(uint64_t n, bool zero) {
    const uint64_t off = (cursor_ + 7) & ~7ull;
    if (img_.size() < off + n) img_.resize(off + n, 0);
    std::memset(img_.data() + off, zero ? 0 : 0xFF, n);
    cursor_ = off + n;
    return off;
}

void FxvolArchive::superblock(uint64_t seq) {
    uint8_t* b = img_.data() + ((seq - 1) & 1ull) * kSuper;
    st<uint32_t>(b, kMagic);
    st<uint32_t>(b + 4, kVersion);
    st<uint64_t>(b + 8, seq);
    st<uint64_t>(b + 16, committed_);
    st<uint32_t>(b + 24, m_.nlods);
    st<uint32_t>(b + 28, m_.dtype);
    for (int a = 0; a < 3; ++a) st<int64_t>(b + 32 + 8 * a, m_.dims[a]);
    st<float>(b + 56, m_.q);
    st<float>(b + 60, m_.hf_exp);
    st<float>(b + 64, m_.dz_frac);
    for (uint64_t l = 0; l < kMaxLod; ++l) st<uint64_t>(b + kLodRootOff + 8 * l, roots_[l]);
    st<uint64_t>(b + kDataOffField, m_.data_off);
    st<uint32_t>(b + kSbCrcLen, crc32c(b, kSbCrcLen));
}

std::string FxvolArchive::put(int lod, int64_t cz, int64_t cy, int64_t cx, const uint8_t* payload, uint64_t len) {
    if (!writable_) return "archive opened read-only";
    if (lod < 0 || lod >= static_cast<int>(kMaxLod)) return "bad lod";
    if (cz < 0 || cy < 0 || cx < 0) return "bad chunk coordinate";
    const uint64_t m = morton3(static_cast<uint64_t>(cz), static_cast<uint64_t>(cy), static_cast<uint64_t>(cx));
    const uint64_t i0 = (m >> 24) & 0xfff, i1 = (m >> 12) & 0xfff, i2 = m & 0xfff;
    // every node of this fresh archive lies past the committed end: no copy-on-write
    if (roots_[lod] == 0) roots_[lod] = alloc(kNodeBytes, true);
    uint64_t l1 = ld<uint64_t>(img_.data() + roots_[lod] + 8 * i0);
    if (l1 == 0) {
        l1 = alloc(kNodeBytes, true);
        st<uint64_t>(img_.data() + roots_[lod] + 8 * i0, l1);
    }
    uint64_t leaf = ld<uint64_t>(img_.data() + l1 + 8 * i1);
    if (leaf == 0) {
        leaf = alloc(kLeafBytes, false);
        st<uint64_t>(img_.data() + l1 + 8 * i1, leaf);
    }
    uint64_t off = 0;
    if (len) {
        off = alloc(len + 4, false);
        std::memcpy(img_.data() + off, payload, len);
        st<uint32_t>(img_.data() + off + len, crc32c(payload, len));
    }
    st<uint64_t>(img_.data() + leaf + 16 * i2, off);
    st<uint64_t>(img_.data() + leaf + 16 * i2 + 8, len);
    return {};
}

std::string FxvolArchive::chunk(int lod, int64_t cz, int64_t cy, int64_t cx, int* coverage, const uint8_t** payload,
                                uint64_t* len) const {
    *coverage = kAbsent;
    *payload = nullptr;
    *len = 0;
    if (lod < 0 || lod >= static_cast<int>(kMaxLod) || cz < 0 || cy < 0 || cx < 0) return {};
    const uint8_t* base = writable_ ? img_.data() : map_;
    const uint64_t hz = writable_ ? cursor_ : hz_;
    const uint64_t root = roots_[lod];
    if (root == 0 || !in_bounds(root, kNodeBytes, hz)) return {};
    const uint64_t m = morton3(static_cast<uint64_t>(cz), static_cast<uint64_t>(cy), static_cast<uint64_t>(cx));
    const uint64_t i0 = (m >> 24) & 0xfff, i1 = (m >> 12) & 0xfff, i2 = m & 0xfff;
    const uint64_t c1 = rd64(root + 8 * i0);
    if (c1 == 0 || !in_bounds(c1, kNodeBytes, hz)) return {};
    const uint64_t c2 = rd64(c1 + 8 * i1);
    if (c2 == 0 || !in_bounds(c2, kLeafBytes, hz)) return {};
    const uint64_t off = ld<uint64_t>(base + c2 + 16 * i2), n = ld<uint64_t>(base + c2 + 16 * i2 + 8);
    if (off == kAbsentOff) return {};
    if (n == 0) {
        *coverage = kZero;
        return {};
    }
    if (off < kDataStart || off > hz || n > hz - off || hz - off - n < 4) return "corrupt chunk offset";
    if (crc32c(base + off, n) != ld<uint32_t>(base + off + n)) return "chunk crc mismatch";
    *coverage = kReal;
    *payload = base + off;
    *len = n;
    return {};
}

std::string FxvolArchive::close() {
    if (!writable_) return {};
    committed_ = cursor_;
    superblock(2);
    writable_ = false;
    FILE* f = std::fopen(path_.c_str(), "wb");
    if (!f) return "cannot write " + path_;
    const bool ok = std::fwrite(img_.data(), 1, committed_, f) == committed_;
    const bool closed = std::fclose(f) == 0;
    img_.clear();
    img_.shrink_to_fit();
    return ok && closed ? std::string() : "cannot write " + path_;
}

}  // namespace fxh
