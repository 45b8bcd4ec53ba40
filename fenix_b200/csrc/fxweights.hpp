// fxweights.hpp — reader for the `.fxweights` flat tensor file (FXWT v1), torch-free.
// Layout (little-endian), as written by the reference's converter and read by its
// load_fxweights (src/ml/weights.hpp:1-10, 63-123):
//   "FXWT" | u32 version | u32 count | u32 reserved
//   count x { u16 name_len | name | u8 dtype | u8 ndim | u64 nbytes | u64 data_off | i64 shape[ndim] }
//   blobs at their data offsets. dtype: 0=f32 1=f16 2=bf16 3=f64 4=i64 5=i32 6=u8 7=i16 8=bool.
// Every field is bounds-checked against the file size, as the reference does. Tensors are
// widened to f32 on load (the net's parameters are f32 in every file this path produces).
#pragma once

#include <cstdint>
#include <cstring>
#include <fstream>
#include <limits>
#include <map>
#include <string>
#include <vector>

namespace fxh {

struct HostTensor {
    std::vector<int64_t> shape;
    std::vector<float> data;
    int64_t numel() const {
        int64_t n = 1;
        for (auto s : shape) n *= s;
        return n;
    }
};

using WeightMap = std::map<std::string, HostTensor>;

inline float half_to_float(uint16_t h) {
    const uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    uint32_t f;
    if (exp == 0) {
        if (man == 0) {
            f = sign << 31;
        } else {  // subnormal
            int e = -1;
            uint32_t m = man;
            do {
                ++e;
                m <<= 1;
            } while ((m & 0x400u) == 0);
            f = (sign << 31) | static_cast<uint32_t>(127 - 15 - e) << 23 | ((m & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        f = (sign << 31) | 0x7f800000u | (man << 13);
    } else {
        f = (sign << 31) | ((exp + 112u) << 23) | (man << 13);
    }
    float out;
    std::memcpy(&out, &f, 4);
    return out;
}

// Returns an empty string on success, else the error message (the caller maps it to a status).
inline std::string load_fxweights(const std::string& path, WeightMap& out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return "fxweights: cannot open " + path;
    std::vector<uint8_t> buf((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    const size_t sz = buf.size();
    const uint8_t* p = buf.data();
    if (sz < 16 || std::memcmp(p, "FXWT", 4) != 0) return "fxweights: bad magic";
    uint32_t version = 0, count = 0;
    std::memcpy(&version, p + 4, 4);
    std::memcpy(&count, p + 8, 4);
    if (version != 1) return "fxweights: unsupported version";
    size_t cur = 16;
    auto have = [&](size_t n) { return cur <= sz && n <= sz - cur; };
    for (uint32_t i = 0; i < count; ++i) {
        uint16_t nlen = 0;
        if (!have(2)) return "fxweights: truncated record header";
        std::memcpy(&nlen, p + cur, 2);
        cur += 2;
        if (!have(nlen)) return "fxweights: truncated record name";
        std::string name(reinterpret_cast<const char*>(p + cur), nlen);
        cur += nlen;
        if (!have(18)) return "fxweights: truncated record for " + name;
        const uint8_t dtype = p[cur], ndim = p[cur + 1];
        cur += 2;
        uint64_t nbytes = 0, off = 0;
        std::memcpy(&nbytes, p + cur, 8);
        std::memcpy(&off, p + cur + 8, 8);
        cur += 16;
        if (!have(size_t{8} * ndim)) return "fxweights: truncated shape for " + name;
        HostTensor t;
        t.shape.resize(ndim);
        for (int d = 0; d < ndim; ++d) {
            std::memcpy(&t.shape[d], p + cur, 8);
            cur += 8;
        }
        size_t isz = 0;
        switch (dtype) {
            case 0: isz = 4; break;
            case 1: case 2: case 7: isz = 2; break;
            case 3: case 4: isz = 8; break;
            case 5: isz = 4; break;
            case 6: case 8: isz = 1; break;
            default: return "fxweights: unknown dtype for " + name;
        }
        if (off > sz || nbytes > sz - off) return "fxweights: blob out of range for " + name;
        uint64_t numel = 1;
        for (auto s : t.shape) {
            if (s < 0 || (s != 0 && numel > std::numeric_limits<uint64_t>::max() / static_cast<uint64_t>(s)))
                return "fxweights: bad shape for " + name;
            numel *= static_cast<uint64_t>(s);
        }
        if (nbytes % isz != 0 || numel != nbytes / isz) return "fxweights: shape/nbytes mismatch for " + name;
        t.data.resize(numel);
        const uint8_t* b = p + off;
        for (uint64_t k = 0; k < numel; ++k) {
            float v = 0.f;
            switch (dtype) {
                case 0: std::memcpy(&v, b + 4 * k, 4); break;
                case 1: { uint16_t h; std::memcpy(&h, b + 2 * k, 2); v = half_to_float(h); } break;
                case 2: { uint16_t h; std::memcpy(&h, b + 2 * k, 2); uint32_t u = static_cast<uint32_t>(h) << 16; std::memcpy(&v, &u, 4); } break;
                case 3: { double d; std::memcpy(&d, b + 8 * k, 8); v = static_cast<float>(d); } break;
                case 4: { int64_t q; std::memcpy(&q, b + 8 * k, 8); v = static_cast<float>(q); } break;
                case 5: { int32_t q; std::memcpy(&q, b + 4 * k, 4); v = static_cast<float>(q); } break;
                case 6: case 8: v = b[k]; break;
                case 7: { int16_t q; std::memcpy(&q, b + 2 * k, 2); v = q; } break;
            }
            t.data[k] = v;
        }
        out.emplace(std::move(name), std::move(t));
    }
    return {};
}

}  // namespace fxh
