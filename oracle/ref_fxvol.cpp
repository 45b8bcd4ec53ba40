// oracle/ref_fxvol.cpp — runs the reference's own .fxvol code (src/codec/dct_block.hpp tile codec,
// src/codec/archive.hpp container) on the CPU, to pin the oracle's C restatement and to write the
// golden fixtures. Test infrastructure: compiled by oracle/Makefile (`make ref`) from the reference
// sources with one substitution, oracle/shim_codec/codec/dct.hpp for the Clang-only DCT-16 panel.
//
//   ref_fxvol enc  <u8|f32> <q> <n> <in.raw> <out.bin>   n 64^3 chunks -> n x [u32 len][payload]
//   ref_fxvol dec  <u8|f32> <q> <in.bin> <out.raw>       n x [u32 len][payload] -> n 64^3 chunks
//   ref_fxvol write <q> <dz> <dy> <dx> <in.raw u8> <out.fxvol>   VolumeArchive create + write_volume + close
//   ref_fxvol read  <in.fxvol> <out.raw u8>                      VolumeArchive open + read_volume_as<u8>(0)
//   ref_fxvol slots <in.fxvol>                                   per LOD / chunk: coverage, offset, length
//
// The decoder's DctParams beyond q (hf_exp, dz_frac, deblock, dc_predict) keep their defaults, as the
// archive reads them (archive.hpp:236-238 stores q, hf_exp, dz_frac; the rest are DctParams{}).
#include "codec/archive.hpp"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

using namespace fenix;
using namespace fenix::codec;

// DctParams with every field a runtime value: a compile-time hf_exp lets the compiler fold the
// step table's std::pow (dct_block.hpp:91-94) at build time, correctly rounded, where libm's powf
// at run time may differ by an ulp; the oracle and the device evaluate powf at run time.
static DctParams params(f32 q) {
    static volatile f32 hf = 0.65f, dz = 0.80f;
    DctParams p{};
    p.q = q;
    p.hf_exp = hf;
    p.dz_frac = dz;
    return p;
}

static std::vector<u8> slurp(const char* path) {
    FILE* f = std::fopen(path, "rb");
    if (!f) {
        std::fprintf(stderr, "cannot open %s\n", path);
        std::exit(2);
    }
    std::fseek(f, 0, SEEK_END);
    const long n = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    std::vector<u8> b(static_cast<usize>(n));
    if (n && std::fread(b.data(), 1, b.size(), f) != b.size()) std::exit(2);
    std::fclose(f);
    return b;
}

static void spit(const char* path, const void* p, usize n) {
    FILE* f = std::fopen(path, "wb");
    if (!f || (n && std::fwrite(p, 1, n, f) != n)) std::exit(2);
    std::fclose(f);
}

template <class T>
static int enc(f32 q, long n, const char* in, const char* out) {
    const usize V = 64 * 64 * 64;
    auto raw = slurp(in);
    if (raw.size() != V * sizeof(T) * static_cast<usize>(n)) return 2;
    std::vector<u8> o;
    for (long i = 0; i < n; ++i) {
        std::span<const T> blk(reinterpret_cast<const T*>(raw.data()) + V * static_cast<usize>(i), V);
        auto p = encode_tile_dct<T>(blk, 4, params(q));
        const u32 len = static_cast<u32>(p.size());
        o.insert(o.end(), reinterpret_cast<const u8*>(&len), reinterpret_cast<const u8*>(&len) + 4);
        o.insert(o.end(), p.begin(), p.end());
    }
    spit(out, o.data(), o.size());
    return 0;
}

template <class T>
static int dec(f32 q, const char* in, const char* out) {
    auto raw = slurp(in);
    std::vector<T> o;
    usize p = 0;
    while (p + 4 <= raw.size()) {
        u32 len;
        std::memcpy(&len, raw.data() + p, 4);
        p += 4;
        if (p + len > raw.size()) return 2;
        auto d = decode_tile_dct<T>(std::span<const u8>(raw.data() + p, len), 4, params(q));
        p += len;
        if (!d) {
            std::fprintf(stderr, "decode error: %s\n", d.error().message.c_str());
            return 3;
        }
        o.insert(o.end(), d->begin(), d->end());
    }
    spit(out, o.data(), o.size() * sizeof(T));
    return 0;
}

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    const std::string cmd = argv[1];
    if (cmd == "enc" && argc == 7) {
        const f32 q = std::strtof(argv[3], nullptr);
        const long n = std::strtol(argv[4], nullptr, 10);
        return std::string(argv[2]) == "f32" ? enc<f32>(q, n, argv[5], argv[6]) : enc<u8>(q, n, argv[5], argv[6]);
    }
    if (cmd == "dec" && argc == 6) {
        const f32 q = std::strtof(argv[3], nullptr);
        return std::string(argv[2]) == "f32" ? dec<f32>(q, argv[4], argv[5]) : dec<u8>(q, argv[4], argv[5]);
    }
    if (cmd == "write" && argc == 8) {
        const f32 q = std::strtof(argv[2], nullptr);
        const Extent3 d{std::atoll(argv[3]), std::atoll(argv[4]), std::atoll(argv[5])};
        auto raw = slurp(argv[6]);
        if (static_cast<s64>(raw.size()) != d.count()) return 2;
        auto a = VolumeArchive::create(argv[7], d, params(q));
        if (!a) return 3;
        VolumeView<const u8> v(raw.data(), d);
        if (auto r = a->write_volume<u8>(v); !r) return 3;
        if (auto r = a->close(); !r) return 3;
        return 0;
    }
    if (cmd == "read" && argc == 4) {
        auto a = VolumeArchive::open(argv[2]);
        if (!a) {
            std::fprintf(stderr, "open error: %s\n", a.error().message.c_str());
            return 3;
        }
        auto v = a->read_volume_as<u8>(0);
        if (!v) {
            std::fprintf(stderr, "read error: %s\n", v.error().message.c_str());
            return 3;
        }
        spit(argv[3], v->data(), static_cast<usize>(v->dims().count()));
        std::printf("%lld %lld %lld %u\n", static_cast<long long>(a->dims().z), static_cast<long long>(a->dims().y),
                    static_cast<long long>(a->dims().x), a->nlods());
        return 0;
    }
    if (cmd == "slots" && argc == 3) {
        auto a = VolumeArchive::open(argv[2]);
        if (!a) return 3;
        for (u32 l = 0; l < a->nlods(); ++l) {
            const ChunkCoord ce = a->chunk_extent(l);
            for (s64 z = 0; z < ce.z; ++z)
                for (s64 y = 0; y < ce.y; ++y)
                    for (s64 x = 0; x < ce.x; ++x)
                        std::printf("%u %lld %lld %lld %d\n", l, static_cast<long long>(z), static_cast<long long>(y),
                                    static_cast<long long>(x), static_cast<int>(a->coverage(l, {z, y, x})));
        }
        return 0;
    }
    std::fprintf(stderr, "usage: see the header of ref_fxvol.cpp\n");
    return 2;
}
