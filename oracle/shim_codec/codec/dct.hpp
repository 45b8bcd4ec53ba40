// oracle/shim_codec/codec/dct.hpp — stands in for the reference's src/codec/dct.hpp when the
// reference's codec headers are compiled with g++ (test infrastructure only). The reference's file
// runs its DCT-16 through a Clang-only vector type (ext_vector_type, dct.hpp:23; g++ rejects its
// scalar initialisers at dct.hpp:121,132), so `-iquote oracle/shim_codec` resolves the
// "codec/dct.hpp" include of src/codec/dct_block.hpp:18 to this file instead.
//
// Same transform as dct.hpp:27-53: the orthonormal DCT-II on 16-point lines, forward X[k] =
// sum_n m[k][n] x[n], inverse (DCT-III) x[n] = sum_k m[k][n] X[k], basis m[k][n] = c_k cos(pi (2n+1)
// k / 32) evaluated in f32 as dct.hpp:43 does, through the even/odd half bases. Scalar, with one
// fixed evaluation order (sequential multiply-then-add, no contraction; 3D passes along x, then y,
// then z) that the oracle's C restatement and the device kernels reproduce, so all three agree
// bit for bit.
#pragma once

#include "core/types.hpp"

#include <span>

namespace fenix::codec {

inline constexpr int kDctN = 16;
inline constexpr int kDctH = kDctN / 2;

struct Dct16Basis {
    f32 me[kDctH][kDctH];  // m[2j][n]
    f32 mo[kDctH][kDctH];  // m[2j+1][n]
};

// The basis values of dct.hpp:37-53 with the cosine correctly rounded (libm's cosf and a compiler's
// compile-time evaluation disagree by an ulp at one argument), written out as literals.
inline const Dct16Basis& dct16_basis() {
    static const Dct16Basis b = {{
        {0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f},
        {0x1.63150ap-2f, 0x1.2d062ep-2f, 0x1.92469ap-3f, 0x1.1a8556p-4f, -0x1.1a855ep-4f, -0x1.9246a2p-3f, -0x1.2d063p-2f, -0x1.63150cp-2f},
        {0x1.4e7ae8p-2f, 0x1.1517a8p-3f, -0x1.1517acp-3f, -0x1.4e7aeap-2f, -0x1.4e7ae8p-2f, -0x1.151798p-3f, 0x1.1517bp-3f, 0x1.4e7aeap-2f},
        {0x1.2d062ep-2f, -0x1.1a855ep-4f, -0x1.63150cp-2f, -0x1.92469p-3f, 0x1.924694p-3f, 0x1.63150ap-2f, 0x1.1a8546p-4f, -0x1.2d0632p-2f},
        {0x1.fffffep-3f, -0x1.fffffep-3f, -0x1.fffffap-3f, 0x1.000006p-2f, 0x1.fffffep-3f, -0x1.00000ap-2f, -0x1.fffff4p-3f, 0x1p-2f},
        {0x1.92469ap-3f, -0x1.63150cp-2f, 0x1.1a8566p-4f, 0x1.2d0628p-2f, -0x1.2d0632p-2f, -0x1.1a84fap-4f, 0x1.63150cp-2f, -0x1.924694p-3f},
        {0x1.1517a8p-3f, -0x1.4e7ae8p-2f, 0x1.4e7aeep-2f, -0x1.1517bep-3f, -0x1.1517bap-3f, 0x1.4e7ae4p-2f, -0x1.4e7aeep-2f, 0x1.1517bep-3f},
        {0x1.1a8556p-4f, -0x1.92469p-3f, 0x1.2d0628p-2f, -0x1.631508p-2f, 0x1.63150ap-2f, -0x1.2d063ap-2f, 0x1.9246c6p-3f, -0x1.1a852p-4f},
    }, {
        {0x1.684b9cp-2f, 0x1.5a730cp-2f, 0x1.3f4a22p-2f, 0x1.17dc14p-2f, 0x1.cb598cp-3f, 0x1.5553ep-3f, 0x1.a46086p-4f, 0x1.1be35p-5f},
        {0x1.5a730cp-2f, 0x1.cb598cp-3f, 0x1.1be33ap-5f, -0x1.5553e8p-3f, -0x1.3f4a22p-2f, -0x1.684b9cp-2f, -0x1.17dc12p-2f, -0x1.a4607ep-4f},
        {0x1.3f4a22p-2f, 0x1.1be35p-5f, -0x1.17dc14p-2f, -0x1.5a730cp-2f, -0x1.a4607ep-4f, 0x1.cb59ap-3f, 0x1.684b9cp-2f, 0x1.5553e8p-3f},
        {0x1.17dc14p-2f, -0x1.5553e8p-3f, -0x1.5a730cp-2f, 0x1.1be388p-5f, 0x1.684b9cp-2f, 0x1.a46062p-4f, -0x1.3f4a2ap-2f, -0x1.cb5998p-3f},
        {0x1.cb598cp-3f, -0x1.3f4a22p-2f, -0x1.a4607ep-4f, 0x1.684b9ep-2f, -0x1.1be36ap-5f, -0x1.5a7306p-2f, 0x1.5553eap-3f, 0x1.17dc0ep-2f},
        {0x1.5553ep-3f, -0x1.684b9cp-2f, 0x1.cb598ep-3f, 0x1.a46062p-4f, -0x1.5a730cp-2f, 0x1.17dc26p-2f, 0x1.1be2ccp-5f, -0x1.3f4a2p-2f},
        {0x1.a46086p-4f, -0x1.17dc16p-2f, 0x1.684b9ap-2f, -0x1.3f4a2ap-2f, 0x1.5553eap-3f, 0x1.1be2ccp-5f, -0x1.cb595ep-3f, 0x1.5a7306p-2f},
        {0x1.1be35p-5f, -0x1.a4607ep-4f, 0x1.5553d4p-3f, -0x1.cb5976p-3f, 0x1.17dc0ep-2f, -0x1.3f4a0cp-2f, 0x1.5a7306p-2f, -0x1.684b9ep-2f},
    }};
    return b;
}

inline void dct16_1d_fwd(const f32* x, f32* X) {
    const Dct16Basis& b = dct16_basis();
    f32 s[kDctH], d[kDctH];
    for (int n = 0; n < kDctH; ++n) {
        s[n] = x[n] + x[kDctN - 1 - n];
        d[n] = x[n] - x[kDctN - 1 - n];
    }
    for (int k = 0; k < kDctH; ++k) {
        f32 e = 0.0f, o = 0.0f;
        for (int n = 0; n < kDctH; ++n) {
            const f32 pe = b.me[k][n] * s[n];
            const f32 po = b.mo[k][n] * d[n];
            e = e + pe;
            o = o + po;
        }
        X[2 * k] = e;
        X[2 * k + 1] = o;
    }
}

inline void dct16_1d_inv(const f32* X, f32* x) {
    const Dct16Basis& b = dct16_basis();
    f32 E[kDctH], O[kDctH];
    for (int n = 0; n < kDctH; ++n) E[n] = O[n] = 0.0f;
    for (int k = 0; k < kDctH; ++k)
        for (int n = 0; n < kDctH; ++n) {
            const f32 pe = b.me[k][n] * X[2 * k];
            const f32 po = b.mo[k][n] * X[2 * k + 1];
            E[n] = E[n] + pe;
            O[n] = O[n] + po;
        }
    for (int n = 0; n < kDctH; ++n) {
        x[n] = E[n] + O[n];
        x[kDctN - 1 - n] = E[n] - O[n];
    }
}

namespace shim_detail {
template <class F>
inline void lines3(f32* d, F&& one) {
    constexpr int N = kDctN;
    f32 in[N], out[N];
    for (int z = 0; z < N; ++z)  // along x
        for (int y = 0; y < N; ++y) {
            f32* p = d + (z * N + y) * N;
            for (int i = 0; i < N; ++i) in[i] = p[i];
            one(in, out);
            for (int i = 0; i < N; ++i) p[i] = out[i];
        }
    for (int z = 0; z < N; ++z)  // along y
        for (int x = 0; x < N; ++x) {
            f32* p = d + z * N * N + x;
            for (int i = 0; i < N; ++i) in[i] = p[i * N];
            one(in, out);
            for (int i = 0; i < N; ++i) p[i * N] = out[i];
        }
    for (int y = 0; y < N; ++y)  // along z
        for (int x = 0; x < N; ++x) {
            f32* p = d + y * N + x;
            for (int i = 0; i < N; ++i) in[i] = p[i * N * N];
            one(in, out);
            for (int i = 0; i < N; ++i) p[i * N * N] = out[i];
        }
}
}  // namespace shim_detail

inline void dct16_3d_fwd(std::span<f32> blk) { shim_detail::lines3(blk.data(), dct16_1d_fwd); }
inline void dct16_3d_inv(std::span<f32> blk) { shim_detail::lines3(blk.data(), dct16_1d_inv); }

}  // namespace fenix::codec
