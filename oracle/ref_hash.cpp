// ref_hash.cpp — prints the reference's own hash64 (src/core/hash.hpp, compiled from the reference
// sources) of a fixed list of byte strings and of a chained 1 MiB-chunk stream, the identity
// hashes of its prediction checkpoints (src/ml/inference.cpp:256-274). Oracle tooling, not product
// code: its output is the golden vector the product's restatement is checked against.
#include "core/hash.hpp"

#include <cstdio>
#include <vector>

int main() {
    // strings of every length class the hash branches on: 0, 1-3, 4-16, > 16 (multiple 16-byte rounds)
    const int lens[] = {0, 1, 2, 3, 4, 7, 8, 15, 16, 17, 31, 32, 33, 100, 4096};
    for (int n : lens) {
        std::vector<fenix::u8> b(static_cast<size_t>(n));
        for (int i = 0; i < n; ++i) b[static_cast<size_t>(i)] = static_cast<fenix::u8>((i * 131 + 7) & 255);
        std::printf("bytes %d %llu %llu\n", n, static_cast<unsigned long long>(fenix::hash64(b)),
                    static_cast<unsigned long long>(fenix::hash64(b, 0x1234567890abcdefULL)));
    }
    // a weights-file-style chained hash over 1 MiB chunks (the last one short)
    std::vector<fenix::u8> chunk(1 << 20);
    fenix::u64 h = 0;
    for (int c = 0; c < 3; ++c) {
        const size_t n = c < 2 ? chunk.size() : 12345;
        for (size_t i = 0; i < n; ++i) chunk[i] = static_cast<fenix::u8>((i * 7 + static_cast<size_t>(c) * 13) & 255);
        h = fenix::hash64({chunk.data(), n}, h);
    }
    std::printf("chain %llu\n", static_cast<unsigned long long>(h));
    return 0;
}
