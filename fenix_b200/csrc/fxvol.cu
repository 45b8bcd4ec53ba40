// fxvol.cu — device .fxvol chunk codec (see fxvol.cuh). Format: src/codec/dct_block.hpp:318-588
// (tile), src/codec/entropy.hpp:61-207 (varints, byte planes, raw bits), src/codec/rans.hpp:22-279.
#include "fxvol.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace fxk {

// The DCT-16 half bases: the reference's formula (dct.hpp:43 — f32 argument pi (2n+1) k / 32, f32
// c_k) with the cosine correctly rounded, written out so every build uses the same values (libm's
// cosf and a compiler's compile-time evaluation disagree by an ulp at one argument).
static const float kMe[8][8] = {
    {0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f},
    {0x1.63150ap-2f, 0x1.2d062ep-2f, 0x1.92469ap-3f, 0x1.1a8556p-4f, -0x1.1a855ep-4f, -0x1.9246a2p-3f, -0x1.2d063p-2f, -0x1.63150cp-2f},
    {0x1.4e7ae8p-2f, 0x1.1517a8p-3f, -0x1.1517acp-3f, -0x1.4e7aeap-2f, -0x1.4e7ae8p-2f, -0x1.151798p-3f, 0x1.1517bp-3f, 0x1.4e7aeap-2f},
    {0x1.2d062ep-2f, -0x1.1a855ep-4f, -0x1.63150cp-2f, -0x1.92469p-3f, 0x1.924694p-3f, 0x1.63150ap-2f, 0x1.1a8546p-4f, -0x1.2d0632p-2f},
    {0x1.fffffep-3f, -0x1.fffffep-3f, -0x1.fffffap-3f, 0x1.000006p-2f, 0x1.fffffep-3f, -0x1.00000ap-2f, -0x1.fffff4p-3f, 0x1p-2f},
    {0x1.92469ap-3f, -0x1.63150cp-2f, 0x1.1a8566p-4f, 0x1.2d0628p-2f, -0x1.2d0632p-2f, -0x1.1a84fap-4f, 0x1.63150cp-2f, -0x1.924694p-3f},
    {0x1.1517a8p-3f, -0x1.4e7ae8p-2f, 0x1.4e7aeep-2f, -0x1.1517bep-3f, -0x1.1517bap-3f, 0x1.4e7ae4p-2f, -0x1.4e7aeep-2f, 0x1.1517bep-3f},
    {0x1.1a8556p-4f, -0x1.92469p-3f, 0x1.2d0628p-2f, -0x1.631508p-2f, 0x1.63150ap-2f, -0x1.2d063ap-2f, 0x1.9246c6p-3f, -0x1.1a852p-4f},
};
static const float kMo[8][8] = {
    {0x1.684b9cp-2f, 0x1.5a730cp-2f, 0x1.3f4a22p-2f, 0x1.17dc14p-2f, 0x1.cb598cp-3f, 0x1.5553ep-3f, 0x1.a46086p-4f, 0x1.1be35p-5f},
    {0x1.5a730cp-2f, 0x1.cb598cp-3f, 0x1.1be33ap-5f, -0x1.5553e8p-3f, -0x1.3f4a22p-2f, -0x1.684b9cp-2f, -0x1.17dc12p-2f, -0x1.a4607ep-4f},
    {0x1.3f4a22p-2f, 0x1.1be35p-5f, -0x1.17dc14p-2f, -0x1.5a730cp-2f, -0x1.a4607ep-4f, 0x1.cb59ap-3f, 0x1.684b9cp-2f, 0x1.5553e8p-3f},
    {0x1.17dc14p-2f, -0x1.5553e8p-3f, -0x1.5a730cp-2f, 0x1.1be388p-5f, 0x1.684b9cp-2f, 0x1.a46062p-4f, -0x1.3f4a2ap-2f, -0x1.cb5998p-3f},
    {0x1.cb598cp-3f, -0x1.3f4a22p-2f, -0x1.a4607ep-4f, 0x1.684b9ep-2f, -0x1.1be36ap-5f, -0x1.5a7306p-2f, 0x1.5553eap-3f, 0x1.17dc0ep-2f},
    {0x1.5553ep-3f, -0x1.684b9cp-2f, 0x1.cb598ep-3f, 0x1.a46062p-4f, -0x1.5a730cp-2f, 0x1.17dc26p-2f, 0x1.1be2ccp-5f, -0x1.3f4a2p-2f},
    {0x1.a46086p-4f, -0x1.17dc16p-2f, 0x1.684b9ap-2f, -0x1.3f4a2ap-2f, 0x1.5553eap-3f, 0x1.1be2ccp-5f, -0x1.cb595ep-3f, 0x1.5a7306p-2f},
    {0x1.1be35p-5f, -0x1.a4607ep-4f, 0x1.5553d4p-3f, -0x1.cb5976p-3f, 0x1.17dc0ep-2f, -0x1.3f4a0cp-2f, 0x1.5a7306p-2f, -0x1.684b9ep-2f},
};

FxvParams fxv_make_params(float q, float hf_exp, float dz_frac) {
    FxvParams p;
    p.q = q;
    p.hf_exp = hf_exp;
    p.dz_frac = dz_frac;
    for (int f = 0; f < 48; ++f) p.stepv[f] = q * std::pow(1.0f + static_cast<float>(f), hf_exp);
    std::memcpy(p.me, kMe, sizeof kMe);
    std::memcpy(p.mo, kMo, sizeof kMo);
    return p;
}

namespace {

constexpr int kV = 4096, kTileV = 64 * 64 * 64, kRawCtx = 24, kMaxCl = 8, kNCat = 18;
constexpr uint32_t kRansL = 1u << 23, kRansScale = 4096;
constexpr int kPad = 16 * 16 * 17;  // padded 16^3 block in shared memory: (z*16 + y)*17 + x
enum { E_TRUNC = 1, E_RANGE = 2, E_UNDERRUN = 3, E_SCRATCH = 4 };

// per-tile work areas of the encoder (worst cases: 64 x 4096 symbols, 16 raw bits each)
constexpr uint64_t kSymCap = 64ull * kV;
constexpr uint64_t kEncCap = 2 * kSymCap + kMaxCl * 128;
constexpr uint64_t kBitsCap = kSymCap * 16 / 8;
constexpr uint64_t kWorkPerTile = kSymCap + kEncCap + kBitsCap;

__device__ __forceinline__ float fm(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fa(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fs(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ int pad_idx(int i) { return (i >> 4) * 17 + (i & 15); }
__device__ __forceinline__ int bitw(uint32_t a) { return a ? 32 - __clz(a) : 0; }
__device__ __forceinline__ int raw_ctx(int fsum, int nsum) {
    return min(3, fsum / 4) * 6 + min(5, nsum);
}

// ---- decode ----------------------------------------------------------------------------------

struct DecHdr {
    int32_t err, K;
    uint32_t nsig_total, bits_n;
    uint64_t bits_off, sym_base, ent_base;
    uint64_t plane_off[kMaxCl];
    uint32_t plane_n[kMaxCl], plane_enc[kMaxCl];
    int32_t dclev[64];
    uint32_t nsig[64];
    uint32_t ncoef[64];
    uint8_t cmap[kRawCtx];
    uint16_t freq[kMaxCl][256];
};

__device__ int dget_var(const uint8_t* b, uint64_t n, uint64_t& p, uint32_t& v) {
    v = 0;
    int sh = 0;
    uint32_t byte;
    do {
        if (p >= n) return E_TRUNC;
        if (sh >= 32) return E_RANGE;
        byte = b[p++];
        v |= (byte & 0x7fu) << sh;
        sh += 7;
    } while (byte & 0x80u);
    return 0;
}

template <class T>
__device__ __forceinline__ int32_t causal_pred(const T* a, int b) {
    const int bz = b >> 4, by = (b >> 2) & 3, bx = b & 3;
    int64_t sum = 0;
    int n = 0;
    if (bx > 0) sum += static_cast<int64_t>(a[b - 1]), ++n;
    if (by > 0) sum += static_cast<int64_t>(a[b - 4]), ++n;
    if (bz > 0) sum += static_cast<int64_t>(a[b - 16]), ++n;
    return n ? static_cast<int32_t>(sum / n) : 0;
}

// One thread per tile: DC / nsig / K / context map / plane headers / bit-stream span
// (dct_block.hpp:494-549, entropy.hpp:115-155).
__global__ void fxv_dec_parse(const uint8_t* __restrict__ blob, const FxvDecTile* __restrict__ tiles, int64_t n,
                              int dc_predict, DecHdr* __restrict__ hdr, unsigned long long* __restrict__ ctr,
                              uint64_t sym_cap, uint64_t ent_cap) {
    const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (t >= n) return;
    DecHdr& h = hdr[t];
    const uint8_t* b = blob + tiles[t].off;
    const uint64_t len = tiles[t].len;
    uint64_t p = 0;
    uint32_t z = 0;
    int e = 0;
    h.K = 0;
    for (int k = 0; k < 64 && !e; ++k) {
        e = dget_var(b, len, p, z);
        if (e) break;
        const int32_t res = static_cast<int32_t>(z >> 1) ^ -static_cast<int32_t>(z & 1u);
        const int32_t pred = dc_predict ? causal_pred(h.dclev, k) : 0;
        h.dclev[k] = static_cast<int32_t>(static_cast<uint32_t>(res) + static_cast<uint32_t>(pred));
    }
    for (int k = 0; k < 64 && !e; ++k) {
        e = dget_var(b, len, p, z);
        if (e) break;
        const int32_t res = static_cast<int32_t>(z >> 1) ^ -static_cast<int32_t>(z & 1u);
        const int32_t pred = dc_predict ? causal_pred(h.nsig, k) : 0;
        const int64_t ns = static_cast<int64_t>(res) + pred;
        if (ns < 0 || ns > kV) e = E_RANGE;
        else h.nsig[k] = static_cast<uint32_t>(ns);
    }
    int K = 0;
    if (!e) {
        if (p >= len) e = E_TRUNC;
        else {
            K = b[p++];
            if (K <= 0 || K > kMaxCl) e = E_RANGE;
        }
    }
    if (!e) {
        if (p + kRawCtx > len) e = E_TRUNC;
        for (int r = 0; r < kRawCtx && !e; ++r) {
            const uint8_t v = b[p++];
            if (v >= K) e = E_RANGE;
            h.cmap[r] = v;
        }
    }
    for (int cl = 0; cl < K && !e; ++cl) {
        uint32_t pn = 0, enc = 0, nused = 0;
        h.plane_n[cl] = 0;
        h.plane_enc[cl] = 0;
        if ((e = dget_var(b, len, p, pn))) break;
        if (pn == 0) continue;
        if (pn > 64u * kV) {
            e = E_RANGE;
            break;
        }
        if ((e = dget_var(b, len, p, enc))) break;
        if ((e = dget_var(b, len, p, nused))) break;
        if (nused > 256) {
            e = E_RANGE;
            break;
        }
        for (int s = 0; s < 256; ++s) h.freq[cl][s] = 0;
        for (uint32_t k = 0; k < nused && !e; ++k) {
            if (p >= len) {
                e = E_TRUNC;
                break;
            }
            const uint8_t s = b[p++];
            uint32_t f = 0;
            if ((e = dget_var(b, len, p, f))) break;
            if (f > 0xffffu) e = E_RANGE;
            else h.freq[cl][s] = static_cast<uint16_t>(f);
        }
        if (e) break;
        uint32_t tot = 0;
        for (int s = 0; s < 256; ++s) tot += h.freq[cl][s];
        if (tot != kRansScale) e = E_RANGE;
        else if (p + enc > len) e = E_TRUNC;
        else {
            h.plane_off[cl] = tiles[t].off + p;
            h.plane_n[cl] = pn;
            h.plane_enc[cl] = enc;
            p += enc;
        }
    }
    uint32_t nb = 0;
    if (!e) e = dget_var(b, len, p, nb);
    if (!e && p + nb > len) e = E_TRUNC;
    if (e) {
        h.err = e;
        return;
    }
    h.K = K;
    h.bits_off = tiles[t].off + p;
    h.bits_n = nb;
    uint64_t sum_n = 0;
    uint32_t ns_tot = 0;
    for (int cl = 0; cl < K; ++cl) sum_n += h.plane_n[cl];
    for (int k = 0; k < 64; ++k) ns_tot += h.nsig[k];
    h.nsig_total = ns_tot;
    h.sym_base = atomicAdd(&ctr[0], static_cast<unsigned long long>(sum_n));
    h.ent_base = atomicAdd(&ctr[1], static_cast<unsigned long long>(ns_tot));
    h.err = (h.sym_base + sum_n > sym_cap || h.ent_base + ns_tot > ent_cap) ? E_SCRATCH : 0;
}

// One warp per category plane (rans.hpp:204-277): the slot table is built in shared memory by the
// warp, then lane 0 runs the (1- or 4-state) decoder over the plane's byte stream.
__global__ void __launch_bounds__(256) fxv_dec_rans(const uint8_t* __restrict__ blob, DecHdr* __restrict__ hdr,
                                                    uint8_t* __restrict__ syms) {
    __shared__ uint8_t slot[kMaxCl][kRansScale];
    __shared__ uint16_t cum[kMaxCl][256];
    DecHdr& h = hdr[blockIdx.x];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (h.err || w >= h.K) return;
    const uint32_t n = h.plane_n[w];
    if (n == 0) return;
    uint32_t f[8], loc = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        f[i] = h.freq[w][lane * 8 + i];
        loc += f[i];
    }
    uint32_t incl = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    uint32_t c = incl - loc;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int s = lane * 8 + i;
        cum[w][s] = static_cast<uint16_t>(c);
        for (uint32_t k = 0; k < f[i]; ++k) slot[w][c + k] = static_cast<uint8_t>(s);
        c += f[i];
    }
    __syncwarp();
    if (lane) return;
    uint64_t base = h.sym_base;
    for (int cl = 0; cl < w; ++cl) base += h.plane_n[cl];
    uint8_t* out = syms + base;
    const uint8_t* st = blob + h.plane_off[w];
    const uint32_t len = h.plane_enc[w];
    if (len == 0) {
        for (uint32_t i = 0; i < n; ++i) out[i] = 0;
        return;
    }
    const uint16_t* fq = h.freq[w];
    uint32_t p = 0;
    bool bad = false;
    auto rd4 = [&]() {
        uint32_t v = kRansL;
        if (p + 4 <= len) {
            v = static_cast<uint32_t>(st[p]) | (static_cast<uint32_t>(st[p + 1]) << 8) |
                (static_cast<uint32_t>(st[p + 2]) << 16) | (static_cast<uint32_t>(st[p + 3]) << 24);
            p += 4;
        }
        return v;
    };
    auto dec = [&](uint32_t& x) -> uint8_t {
        const uint32_t s = slot[w][x & (kRansScale - 1)];
        x = static_cast<uint32_t>(fq[s]) * (x >> 12) + (x & (kRansScale - 1)) - cum[w][s];
        while (x < kRansL && p < len) x = (x << 8) | st[p++];
        bad |= s >= kNCat;
        return static_cast<uint8_t>(s);
    };
    if (n < 4096) {
        uint32_t x0 = rd4();
        for (uint32_t i = 0; i < n; ++i) out[i] = dec(x0);
    } else {
        uint32_t x0 = rd4(), x1 = rd4(), x2 = rd4(), x3 = rd4();
        const uint32_t ng = n / 4, base4 = ng * 4;
        for (uint32_t g = 0; g < ng; ++g) {
            out[4 * g] = dec(x0);
            out[4 * g + 1] = dec(x1);
            out[4 * g + 2] = dec(x2);
            out[4 * g + 3] = dec(x3);
        }
        for (uint32_t i = base4; i < n; ++i) {
            uint32_t& x = (i & 3) == 0 ? x0 : (i & 3) == 1 ? x1 : (i & 3) == 2 ? x2 : x3;
            out[i] = dec(x);
        }
    }
    if (bad) atomicExch(&h.err, static_cast<int32_t>(E_RANGE));
}

constexpr int kWalkTiles = 32;

// One thread per tile (dct_block.hpp:556-570): the significance context picks the clustered stream
// of each coefficient in scan order; magnitudes and signs come from the shared raw bit stream.
// Nonzero coefficients go to `ent` as (index, value) pairs, block b's from ent_base + sum(nsig[<b]).
__global__ void __launch_bounds__(kWalkTiles) fxv_dec_walk(const uint8_t* __restrict__ blob, DecHdr* __restrict__ hdr,
                                                          const uint8_t* __restrict__ syms,
                                                          const uint32_t* __restrict__ scan_g, FxvParams P,
                                                          float2* __restrict__ ent, int64_t n) {
    extern __shared__ uint32_t dsm[];
    uint32_t* scan = dsm;                    // [4096] packed idx | fsum << 16 | edge << 24
    uint32_t* sigw = dsm + kV;               // [tiles per CTA][257] 2-bit significance
    __shared__ float stepv[48];
    __shared__ uint8_t cmaps[kWalkTiles][kRawCtx];
    for (int k = threadIdx.x; k < kV; k += blockDim.x) scan[k] = scan_g[k];
    for (int k = threadIdx.x; k < 48; k += blockDim.x) stepv[k] = P.stepv[k];
    __syncthreads();
    const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (t >= n) return;
    DecHdr& h = hdr[t];
    if (h.err) return;
    uint32_t* sg = sigw + threadIdx.x * 257;
    uint8_t* cm = cmaps[threadIdx.x];
    for (int r = 0; r < kRawCtx; ++r) cm[r] = h.cmap[r];
    uint32_t cur[kMaxCl], pn[kMaxCl];
    uint64_t pb[kMaxCl];
    uint64_t base = h.sym_base;
    for (int cl = 0; cl < kMaxCl; ++cl) {
        cur[cl] = 0;
        pn[cl] = cl < h.K ? h.plane_n[cl] : 0;
        pb[cl] = base;
        base += pn[cl];
    }
    const uint8_t* bp = blob + h.bits_off;
    const uint32_t bn = h.bits_n;
    uint32_t bpos = 0;
    uint64_t acc = 0;
    int nb = 0;
    auto get = [&](int bits) -> uint32_t {
        if (bits <= 0) return 0;
        while (nb < bits) {
            acc |= static_cast<uint64_t>(bpos < bn ? bp[bpos++] : 0) << nb;
            nb += 8;
        }
        const uint32_t v = static_cast<uint32_t>(acc & ((1u << bits) - 1u));
        acc >>= bits;
        nb -= bits;
        return v;
    };
    auto sig = [&](int i) -> int { return (sg[i >> 4] >> ((i & 15) * 2)) & 3; };
    const float dz = P.dz_frac;
    uint64_t eb = h.ent_base;
    for (int b = 0; b < 64; ++b) {
        for (int w = 0; w < 256; ++w) sg[w] = 0;
        const uint32_t ns = h.nsig[b];
        uint32_t cnt = 0;
        for (uint32_t pos = 0; pos < ns; ++pos) {
            const uint32_t e = scan[pos];
            const int i = e & 0xffff, fsum = (e >> 16) & 0xff, edge = e >> 24;
            const int nsum = ((edge & 1) ? sig(i - 256) : 0) + ((edge & 2) ? sig(i - 16) : 0) + ((edge & 4) ? sig(i - 1) : 0);
            const int cl = cm[raw_ctx(fsum, nsum)];
            if (cur[cl] >= pn[cl]) {
                h.err = E_UNDERRUN;
                return;
            }
            const int cat = syms[pb[cl] + cur[cl]++];
            if (cat > 0) {
                const uint32_t a = (1u << (cat - 1)) + get(cat - 1);
                const bool neg = get(1) != 0;
                const float mag = fm(stepv[fsum], fa(fa(fs(static_cast<float>(a), 1.0f), dz), 0.40f));
                ent[eb + cnt++] = make_float2(__int_as_float(i), neg ? -mag : mag);
                sg[i >> 4] |= static_cast<uint32_t>(a < 3 ? a : 3) << ((i & 15) * 2);
            }
        }
        h.ncoef[b] = cnt;
        eb += ns;
    }
}

// 16-point DCT-III on a line in shared memory (dct.hpp:71-88 via the even/odd half bases)
__device__ __forceinline__ void inv_line(const float (*me)[8], const float (*mo)[8], const float* x, float* out) {
    float E[8], O[8];
#pragma unroll
    for (int n = 0; n < 8; ++n) E[n] = O[n] = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float xe = x[2 * k], xo = x[2 * k + 1];
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            E[n] = fa(E[n], fm(me[k][n], xe));
            O[n] = fa(O[n], fm(mo[k][n], xo));
        }
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
        out[n] = fa(E[n], O[n]);
        out[15 - n] = fs(E[n], O[n]);
    }
}

// 16-point DCT-II (dct.hpp:55-69)
__device__ __forceinline__ void fwd_line(const float (*me)[8], const float (*mo)[8], const float* x, float* out) {
    float s[8], d[8];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
        s[n] = fa(x[n], x[15 - n]);
        d[n] = fs(x[n], x[15 - n]);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        float e = 0.0f, o = 0.0f;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            e = fa(e, fm(me[k][n], s[n]));
            o = fa(o, fm(mo[k][n], d[n]));
        }
        out[2 * k] = e;
        out[2 * k + 1] = o;
    }
}

// deblock filter on one boundary line (dct_block.hpp:275-287); R is the tile's f32 reconstruction
__device__ __forceinline__ void db_line(float* R, int base, int st, float beta, float tc) {
    const float p2 = R[base - 3 * st], p1 = R[base - 2 * st], p0 = R[base - st], q0 = R[base], q1 = R[base + st],
                q2 = R[base + 2 * st];
    const float dp = fabsf(fa(fs(p2, fm(2.0f, p1)), p0)), dq = fabsf(fa(fs(q2, fm(2.0f, q1)), q0));
    if (fa(dp, dq) >= beta) return;
    float delta = fm(fs(fm(9.0f, fs(q0, p0)), fm(3.0f, fs(q1, p1))), 0.0625f);
    if (fabsf(delta) >= fm(10.0f, tc)) return;
    delta = delta < -tc ? -tc : (tc < delta ? tc : delta);
    R[base - st] = fa(p0, delta);
    R[base] = fs(q0, delta);
}

// The reference filters boundary b with one raster walk over (i, j), each step the z-, y- then
// x-edge line. Lines that meet no other line run in any order; those that meet fall into groups
// that never meet each other — per x column outside the band (z/y lines), per y row (z/x lines),
// per z slice (y/x lines), and the band cube — each run in the reference's order.
__device__ void deblock_phase(float* R, int b, float beta, float tc) {
    const int lo = b - 3, hi = b + 2;
    auto nbi = [&](int k) { return k < lo ? k : k + 6; };
    auto Z = [&](int i, int j) { db_line(R, (b * 64 + i) * 64 + j, 4096, beta, tc); };
    auto Y = [&](int i, int j) { db_line(R, (i * 64 + b) * 64 + j, 64, beta, tc); };
    auto X = [&](int i, int j) { db_line(R, (i * 64 + j) * 64 + b, 1, beta, tc); };
    constexpr int kFree = 58 * 58 * 3, kGroups = 1 + 3 * 58;
    for (int it = threadIdx.x; it < kFree + kGroups; it += blockDim.x) {
        if (it == 0) {
            for (int i = lo; i <= hi; ++i)
                for (int j = lo; j <= hi; ++j) {
                    Z(i, j);
                    Y(i, j);
                    X(i, j);
                }
        } else if (it < kGroups) {
            const int g = it - 1, kind = g / 58, c = nbi(g % 58);
            if (kind == 0) {
                for (int i = lo; i <= hi; ++i) {
                    Z(i, c);
                    Y(i, c);
                }
            } else if (kind == 1) {
                for (int i = lo; i <= hi && i < c; ++i) X(i, c);
                for (int j = lo; j <= hi; ++j) Z(c, j);
                for (int i = max(lo, c + 1); i <= hi; ++i) X(i, c);
            } else {
                for (int j = lo; j <= hi; ++j) {
                    Y(c, j);
                    X(c, j);
                }
            }
        } else {
            const int k = it - kGroups, pr = k / 3, op = k % 3, i = nbi(pr / 58), j = nbi(pr % 58);
            if (op == 0) Z(i, j);
            else if (op == 1) Y(i, j);
            else X(i, j);
        }
    }
}

// One CTA per tile (dct_block.hpp:552-587): inverse DCT of the 64 blocks (two at a time) into the
// tile's f32 reconstruction, deblocking, then u8 rounding (dtype.hpp:50-55) into the destination.
__global__ void __launch_bounds__(512) fxv_dec_recon(const DecHdr* __restrict__ hdr, const float2* __restrict__ ent,
                                                     FxvParams P, float* __restrict__ recon, int64_t t0,
                                                     const FxvDecTile* __restrict__ tiles, uint8_t* __restrict__ out,
                                                     int64_t dz, int64_t dy, int64_t dx) {
    __shared__ float blk[2][kPad];
    __shared__ uint32_t pre[65];
    __shared__ float me[8][8], mo[8][8];
    const int64_t t = t0 + blockIdx.x;
    const DecHdr& h = hdr[t];
    if (h.err) return;
    float* R = recon + static_cast<int64_t>(blockIdx.x) * kTileV;
    if (threadIdx.x == 0) {
        pre[0] = 0;
        for (int b = 0; b < 64; ++b) pre[b + 1] = pre[b] + h.nsig[b];
    }
    if (threadIdx.x < 64) me[threadIdx.x >> 3][threadIdx.x & 7] = P.me[threadIdx.x >> 3][threadIdx.x & 7];
    else if (threadIdx.x < 128) mo[(threadIdx.x - 64) >> 3][threadIdx.x & 7] = P.mo[(threadIdx.x - 64) >> 3][threadIdx.x & 7];
    __syncthreads();
    const int half = threadIdx.x >> 8, lt = threadIdx.x & 255;
    float* B = blk[half];
    const float dcs = fm(P.q, 0.0625f);
    for (int bb = 0; bb < 32; ++bb) {
        const int b = 2 * bb + half, bz = b >> 4, by = (b >> 2) & 3, bx = b & 3;
        for (int k = lt; k < kPad; k += 256) B[k] = 0.0f;
        __syncthreads();
        const float2* E = ent + h.ent_base + pre[b];
        const uint32_t nc = h.ncoef[b];
        for (uint32_t k = lt; k < nc; k += 256) {
            const float2 v = E[k];
            B[pad_idx(__float_as_int(v.x))] = v.y;
        }
        __syncthreads();
        float x[16], y[16];
        {  // along x: line (z, y) = lt
            float* L = B + lt * 17;
#pragma unroll
            for (int i = 0; i < 16; ++i) x[i] = L[i];
            inv_line(me, mo, x, y);
#pragma unroll
            for (int i = 0; i < 16; ++i) L[i] = y[i];
        }
        __syncthreads();
        {  // along y: line (z, x)
            float* L = B + (lt >> 4) * 16 * 17 + (lt & 15);
#pragma unroll
            for (int i = 0; i < 16; ++i) x[i] = L[i * 17];
            inv_line(me, mo, x, y);
#pragma unroll
            for (int i = 0; i < 16; ++i) L[i * 17] = y[i];
        }
        __syncthreads();
        {  // along z: line (y, x), + DC, to the tile
            const int yy = lt >> 4, xx = lt & 15;
            const float* L = B + yy * 17 + xx;
#pragma unroll
            for (int i = 0; i < 16; ++i) x[i] = L[i * 16 * 17];
            inv_line(me, mo, x, y);
            const float dc = fm(static_cast<float>(h.dclev[b]), dcs);
            float* o = R + ((bz * 16) * 64 + by * 16 + yy) * 64 + bx * 16 + xx;
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i * 4096] = fa(y[i], dc);
        }
        __syncthreads();
    }
    const float tc = fm(P.deblock_tc, P.q), beta = fm(P.deblock_beta, P.q);
    if (P.deblock && tc > 0.0f) {
        for (int b = 16; b < 64; b += 16) {
            deblock_phase(R, b, beta, tc);
            __syncthreads();
        }
    }
    if (!out) return;
    const int64_t z0 = tiles[t].z0, y0 = tiles[t].y0, x0 = tiles[t].x0;
    for (int v = threadIdx.x; v < kTileV; v += blockDim.x) {
        const int64_t gz = z0 + (v >> 12), gy = y0 + ((v >> 6) & 63), gx = x0 + (v & 63);
        if (gz >= dz || gy >= dy || gx >= dx) continue;
        float r = rintf(R[v]);
        r = r < 0.0f ? 0.0f : (r > 255.0f ? 255.0f : r);
        out[(gz * dy + gy) * dx + gx] = static_cast<uint8_t>(r);
    }
}

// ---- encode ----------------------------------------------------------------------------------

struct EncBlk {
    int32_t dclev;
    uint32_t nsig;
    uint32_t cnt[kMaxCl + 1];  // symbols per cluster, raw bits (last)
    uint32_t off[kMaxCl + 1];  // their offsets within the tile's planes / bit stream
};

struct EncHdr {
    int32_t nonzero, K, err, pad;
    uint32_t hist[kRawCtx * kNCat];
    uint8_t cmap[kRawCtx];
    float bc[kMaxCl][kNCat];
    uint32_t plane_n[kMaxCl];
    uint32_t cc[kMaxCl][kNCat];  // category counts per cluster plane
    uint32_t freq[kMaxCl][kNCat];
    uint32_t enc_start[kMaxCl], enc_len[kMaxCl];
    uint64_t enc_off[kMaxCl];
    uint32_t nbits;
};

struct EncOut {
    uint64_t off;
    uint32_t len, err;
};

// One CTA per 16^3 block (dct_block.hpp:131-168, archive.hpp:792-811 edge replication).
template <bool F32>
__global__ void __launch_bounds__(256) fxv_enc_quant(const uint8_t* __restrict__ src8, const float* __restrict__ src32,
                                                     int64_t dz, int64_t dy, int64_t dx,
                                                     const FxvEncTile* __restrict__ tiles, FxvParams P,
                                                     const uint16_t* __restrict__ rank, int16_t* __restrict__ lev,
                                                     float* __restrict__ coef, EncBlk* __restrict__ blk,
                                                     EncHdr* __restrict__ eh, int encode_all) {
    __shared__ float c[kPad];
    __shared__ float me[8][8], mo[8][8];
    __shared__ int red_i[8];
    __shared__ unsigned red_n[8];
    __shared__ float s_dcv;
    __shared__ int s_dl;
    const int b = blockIdx.x, lt = threadIdx.x, lane = lt & 31, wid = lt >> 5;
    const int64_t t = blockIdx.y;
    const int bz = b >> 4, by = (b >> 2) & 3, bx = b & 3;
    if (lt < 64) me[lt >> 3][lt & 7] = P.me[lt >> 3][lt & 7];
    else if (lt < 128) mo[(lt - 64) >> 3][lt & 7] = P.mo[(lt - 64) >> 3][lt & 7];
    const int64_t oz = tiles[t].z0 + bz * 16, oy = tiles[t].y0 + by * 16, ox = tiles[t].x0 + bx * 16;
    int isum = 0;
    unsigned nz = 0;
    for (int k = lt; k < kV; k += 256) {
        const int z = k >> 8, y = (k >> 4) & 15, x = k & 15;
        const int64_t gz = min(oz + z, dz - 1), gy = min(oy + y, dy - 1), gx = min(ox + x, dx - 1);
        const int64_t gi = (gz * dy + gy) * dx + gx;
        float v;
        if constexpr (F32) {
            v = src32[gi];
        } else {
            const int u = src8[gi];
            isum += u;
            v = static_cast<float>(u);
        }
        nz |= v != 0.0f;
        c[pad_idx(k)] = v;
    }
    for (int o = 16; o > 0; o >>= 1) {
        isum += __shfl_xor_sync(0xffffffffu, isum, o);
        nz |= __shfl_xor_sync(0xffffffffu, nz, o);
    }
    if (lane == 0) {
        red_i[wid] = isum;
        red_n[wid] = nz;
    }
    __syncthreads();
    if (lt == 0) {
        double msum = 0;
        unsigned anz = 0;
        for (int w = 0; w < 8; ++w) anz |= red_n[w];
        if constexpr (F32) {
            for (int k = 0; k < kV; ++k) msum = __dadd_rn(msum, static_cast<double>(c[pad_idx(k)]));
        } else {
            int s = 0;
            for (int w = 0; w < 8; ++w) s += red_i[w];
            msum = static_cast<double>(s);
        }
        if (anz || encode_all) atomicOr(&eh[t].nonzero, 1);
        const float dc_step = fm(P.q, 0.0625f);
        const float mean = static_cast<float>(__ddiv_rn(msum, 4096.0));
        const int dl = static_cast<int>(lroundf(__fdiv_rn(mean, dc_step)));
        s_dl = dl;
        s_dcv = fm(static_cast<float>(dl), dc_step);
    }
    __syncthreads();
    const float dcv = s_dcv;
    for (int k = lt; k < kV; k += 256) {
        const int pi = pad_idx(k);
        c[pi] = fs(c[pi], dcv);
    }
    __syncthreads();
    float x[16], y[16];
    {  // along x
        float* L = c + lt * 17;
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] = L[i];
        fwd_line(me, mo, x, y);
#pragma unroll
        for (int i = 0; i < 16; ++i) L[i] = y[i];
    }
    __syncthreads();
    {  // along y
        float* L = c + (lt >> 4) * 16 * 17 + (lt & 15);
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] = L[i * 17];
        fwd_line(me, mo, x, y);
#pragma unroll
        for (int i = 0; i < 16; ++i) L[i * 17] = y[i];
    }
    __syncthreads();
    {  // along z
        float* L = c + (lt >> 4) * 17 + (lt & 15);
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] = L[i * 16 * 17];
        fwd_line(me, mo, x, y);
#pragma unroll
        for (int i = 0; i < 16; ++i) L[i * 16 * 17] = y[i];
    }
    __syncthreads();
    const int64_t bo = (t * 64 + b) * static_cast<int64_t>(kV);
    const float omd = fs(1.0f, P.dz_frac);
    int maxr = -1;
    for (int k = lt; k < kV; k += 256) {
        const int z = k >> 8, y2 = (k >> 4) & 15, x2 = k & 15;
        const float v = c[pad_idx(k)];
        const float step = P.stepv[z + y2 + x2], a0 = fabsf(v);
        coef[bo + k] = v;
        int level = 0;
        if (a0 >= fm(P.dz_frac, step)) {
            const float tq = fa(__fdiv_rn(a0, step), omd);
            level = (v < 0.0f ? -1 : 1) * static_cast<int>(floorf(tq));
        }
        level = level < -32768 ? -32768 : (level > 32767 ? 32767 : level);
        lev[bo + k] = static_cast<int16_t>(level);
        if (level != 0) maxr = max(maxr, static_cast<int>(rank[k]));
    }
    for (int o = 16; o > 0; o >>= 1) maxr = max(maxr, __shfl_xor_sync(0xffffffffu, maxr, o));
    if (lane == 0) red_i[wid] = maxr;
    __syncthreads();
    if (lt == 0) {
        int m = -1;
        for (int w = 0; w < 8; ++w) m = max(m, red_i[w]);
        blk[t * 64 + b].dclev = s_dl;
        blk[t * 64 + b].nsig = static_cast<uint32_t>(m + 1);
    }
}

__device__ __forceinline__ int nsum_lev(const int16_t* L, int i, int edge) {
    auto s = [&](int k) { const int a = abs(static_cast<int>(L[k])); return a < 3 ? a : 3; };
    return ((edge & 1) ? s(i - 256) : 0) + ((edge & 2) ? s(i - 16) : 0) + ((edge & 4) ? s(i - 1) : 0);
}

// Raw-context histogram of the quantised levels (dct_block.hpp:336-347): every coefficient's
// neighbours precede it in the scan, so its context depends only on the final neighbour levels.
__global__ void __launch_bounds__(256) fxv_enc_hist(const int16_t* __restrict__ lev, const EncBlk* __restrict__ blk,
                                                    const uint32_t* __restrict__ scan, EncHdr* __restrict__ eh) {
    __shared__ uint32_t h[kRawCtx * kNCat];
    const int b = blockIdx.x;
    const int64_t t = blockIdx.y;
    for (int k = threadIdx.x; k < kRawCtx * kNCat; k += 256) h[k] = 0;
    __syncthreads();
    if (!eh[t].nonzero) return;
    const uint32_t ns = blk[t * 64 + b].nsig;
    const int16_t* L = lev + (t * 64 + b) * static_cast<int64_t>(kV);
    for (uint32_t pos = threadIdx.x; pos < ns; pos += 256) {
        const uint32_t e = scan[pos];
        const int i = e & 0xffff, fsum = (e >> 16) & 0xff, edge = e >> 24;
        const int cat = bitw(static_cast<uint32_t>(abs(static_cast<int>(L[i]))));
        atomicAdd(&h[raw_ctx(fsum, nsum_lev(L, i, edge)) * kNCat + cat], 1u);
    }
    __syncthreads();
    for (int k = threadIdx.x; k < kRawCtx * kNCat; k += 256)
        if (h[k]) atomicAdd(&eh[t].hist[k], h[k]);
}

// log2 x = e + 2 atanh((m-1)/(m+1)) / ln 2 with m in [sqrt(1/2), sqrt(2)) (series to t^23): the
// same operations as the CPU restatement's portable log2, so both pick the same clusters.
__device__ double log2s(double x) {
    int e;
    double m = frexp(x, &e);
    if (m < 0.70710678118654752440) {
        m = m * 2.0;
        e -= 1;
    }
    const double t = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0)), t2 = __dmul_rn(t, t);
    double s = __ddiv_rn(1.0, 23.0);
    for (int k = 10; k >= 0; --k) s = __dadd_rn(__dmul_rn(s, t2), __ddiv_rn(1.0, static_cast<double>(2 * k + 1)));
    const double ln_m = __dmul_rn(__dmul_rn(2.0, t), s);
    return __dadd_rn(static_cast<double>(e), __dmul_rn(ln_m, 1.4426950408889634));
}

__device__ double clust_cost(const uint32_t* a, const uint32_t* b) {
    double n = 0;
    int nused = 0;
    for (int c = 0; c < kNCat; ++c) {
        const uint32_t h = a[c] + (b ? b[c] : 0u);
        n = __dadd_rn(n, static_cast<double>(h));
        nused += h != 0;
    }
    if (n == 0) return 0.0;
    double ent = 0;
    for (int c = 0; c < kNCat; ++c) {
        const uint32_t h = a[c] + (b ? b[c] : 0u);
        if (h) ent = __dadd_rn(ent, __dmul_rn(static_cast<double>(h), log2s(__ddiv_rn(n, static_cast<double>(h)))));
    }
    return __dadd_rn(__dadd_rn(ent, __dmul_rn(static_cast<double>(nused), 16.0)), 24.0);
}

// Greedy context clustering (dct_block.hpp:171-257), one warp per tile: every candidate pair's
// merged cost is cached and only the pairs of the merged cluster are re-evaluated; the winner is
// the first minimum in (i, j) order, as the reference's scan picks it. Then RDOQ's per-cluster
// category costs (dct_block.hpp:358-371).
__global__ void __launch_bounds__(32) fxv_enc_cluster(EncHdr* __restrict__ eh) {
    __shared__ uint32_t ch[kRawCtx][kNCat];
    __shared__ double ccost[kRawCtx], pc[kRawCtx * kRawCtx];
    __shared__ int alive[kRawCtx];
    __shared__ uint8_t clo[kRawCtx];
    __shared__ int s_nact;
    EncHdr& h = eh[blockIdx.x];
    const int lane = threadIdx.x;
    if (!h.nonzero) return;
    for (int k = lane; k < kRawCtx * kNCat; k += 32) ch[k / kNCat][k % kNCat] = h.hist[k];
    __syncwarp();
    if (lane < kRawCtx) {
        uint32_t tot = 0;
        for (int c = 0; c < kNCat; ++c) tot += ch[lane][c];
        alive[lane] = tot > 0;
        ccost[lane] = tot > 0 ? clust_cost(ch[lane], nullptr) : 0.0;
        clo[lane] = static_cast<uint8_t>(lane);
    }
    __syncwarp();
    if (lane == 0) {
        int na = 0;
        for (int r = 0; r < kRawCtx; ++r) na += alive[r];
        s_nact = na;
    }
    __syncwarp();
    int nact = s_nact;
    for (int p = lane; p < kRawCtx * kRawCtx; p += 32) {
        const int i = p / kRawCtx, j = p % kRawCtx;
        if (i < j && alive[i] && alive[j]) pc[p] = clust_cost(ch[i], ch[j]);
    }
    __syncwarp();
    while (nact > 1) {
        const bool force = nact > kMaxCl;
        double bd = 0;
        int bp = 1 << 30;
        for (int p = lane; p < kRawCtx * kRawCtx; p += 32) {
            const int i = p / kRawCtx, j = p % kRawCtx;
            if (!(i < j && alive[i] && alive[j])) continue;
            const double d = __dsub_rn(__dsub_rn(pc[p], ccost[i]), ccost[j]);
            if (bp == (1 << 30) || d < bd) {
                bd = d;
                bp = p;
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const double od = __shfl_xor_sync(0xffffffffu, bd, o);
            const int op = __shfl_xor_sync(0xffffffffu, bp, o);
            if (op != (1 << 30) && (bp == (1 << 30) || od < bd || (od == bd && op < bp))) {
                bd = od;
                bp = op;
            }
        }
        if (bp == (1 << 30) || (!force && bd >= 0)) break;
        const int bi = bp / kRawCtx, bj = bp % kRawCtx;
        if (lane < kNCat) ch[bi][lane] += ch[bj][lane];
        __syncwarp();
        if (lane == 0) {
            ccost[bi] = clust_cost(ch[bi], nullptr);
            alive[bj] = 0;
            for (int r = 0; r < kRawCtx; ++r)
                if (clo[r] == bj) clo[r] = static_cast<uint8_t>(bi);
        }
        __syncwarp();
        --nact;
        if (lane < kRawCtx && lane != bi && alive[lane]) {
            const int i = min(bi, lane), j = max(bi, lane);
            pc[i * kRawCtx + j] = clust_cost(ch[i], ch[j]);
        }
        __syncwarp();
    }
    if (lane == 0) {
        int remap[kRawCtx];
        for (int r = 0; r < kRawCtx; ++r) remap[r] = -1;
        int K = 0;
        if (s_nact == 0) {
            for (int r = 0; r < kRawCtx; ++r) clo[r] = 0;
            K = 1;
        } else {
            for (int r = 0; r < kRawCtx; ++r)
                if (alive[clo[r]] && remap[clo[r]] < 0) remap[clo[r]] = K++;
            if (K == 0) K = 1;
            for (int r = 0; r < kRawCtx; ++r) clo[r] = static_cast<uint8_t>(alive[clo[r]] ? remap[clo[r]] : 0);
        }
        h.K = K;
        for (int r = 0; r < kRawCtx; ++r) h.cmap[r] = clo[r];
    }
    __syncwarp();
    const int K = h.K;
    for (int k = lane; k < K * kNCat; k += 32) {
        const int cl = k / kNCat, cat = k % kNCat;
        double tot = 0, v = 0;
        for (int c = 0; c < kNCat; ++c) {
            double s = 0;
            for (int r = 0; r < kRawCtx; ++r)
                if (clo[r] == cl) s = __dadd_rn(s, static_cast<double>(h.hist[r * kNCat + c]));
            tot = __dadd_rn(tot, s);
            if (c == cat) v = s;
        }
        h.bc[cl][cat] = static_cast<float>(-log2s(__ddiv_rn(__dadd_rn(v, 0.5), __dadd_rn(tot, 0.5 * kNCat))));
    }
}

// RDOQ (dct_block.hpp:372-412), one CTA per block. The reference decides in scan order; every
// coefficient's causal neighbours lie in the previous frequency shell (z+y+x one less), so the
// decisions of one shell are independent and a shell is decided in parallel, shell after shell.
__global__ void __launch_bounds__(128) fxv_enc_rdoq(int16_t* __restrict__ lev, const float* __restrict__ coef,
                                                    EncBlk* __restrict__ blk, const uint32_t* __restrict__ scan,
                                                    const uint16_t* __restrict__ shell, const EncHdr* __restrict__ eh,
                                                    FxvParams P) {
    __shared__ float bc[kMaxCl][kNCat];
    __shared__ uint8_t cmap[kRawCtx];
    __shared__ float stepv[48];
    __shared__ int red[4];
    const int b = blockIdx.x;
    const int64_t t = blockIdx.y;
    const EncHdr& h = eh[t];
    if (!h.nonzero) return;
    for (int k = threadIdx.x; k < kMaxCl * kNCat; k += 128) bc[k / kNCat][k % kNCat] = h.bc[k / kNCat][k % kNCat];
    for (int k = threadIdx.x; k < kRawCtx; k += 128) cmap[k] = h.cmap[k];
    for (int k = threadIdx.x; k < 48; k += 128) stepv[k] = P.stepv[k];
    __syncthreads();
    int16_t* L = lev + (t * 64 + b) * static_cast<int64_t>(kV);
    const float* C = coef + (t * 64 + b) * static_cast<int64_t>(kV);
    const uint32_t ns = blk[t * 64 + b].nsig;
    const float dz = P.dz_frac, lamq = P.rdoq_lambda;
    for (int f = 0; f < 46; ++f) {
        const uint32_t s0 = shell[f];
        if (s0 >= ns) break;
        const uint32_t s1 = min(static_cast<uint32_t>(shell[f + 1]), ns);
        for (uint32_t pos = s0 + threadIdx.x; pos < s1; pos += 128) {
            const uint32_t e = scan[pos];
            const int i = e & 0xffff, fsum = (e >> 16) & 0xff, edge = e >> 24;
            const int l = L[i];
            const uint32_t m0 = static_cast<uint32_t>(abs(l));
            if (m0 == 0) continue;
            const int cl = cmap[raw_ctx(fsum, nsum_lev(L, i, edge))];
            const float s = stepv[fsum], lam = fm(fm(lamq, s), s), ac = fabsf(C[i]);
            auto rd = [&](uint32_t m) {
                const float dq = m ? fm(s, fa(fa(fs(static_cast<float>(m), 1.0f), dz), 0.40f)) : 0.0f;
                const int cat = m ? bitw(m) : 0;
                const float df = fs(ac, dq);
                return fa(fm(df, df), fm(lam, fa(bc[cl][cat], static_cast<float>(m ? cat : 0))));
            };
            uint32_t bm = m0;
            float best = rd(m0);
            const float c0 = rd(0);
            if (c0 < best) {
                best = c0;
                bm = 0;
            }
            if (m0 >= 2) {
                const float c1 = rd(m0 - 1);
                if (c1 < best) {
                    best = c1;
                    bm = m0 - 1;
                }
            }
            L[i] = static_cast<int16_t>(l < 0 ? -static_cast<int>(bm) : static_cast<int>(bm));
        }
        __syncthreads();
    }
    int m = -1;
    for (uint32_t pos = threadIdx.x; pos < ns; pos += 128)
        if (L[scan[pos] & 0xffff] != 0) m = max(m, static_cast<int>(pos));
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) blk[t * 64 + b].nsig = static_cast<uint32_t>(max(max(red[0], red[1]), max(red[2], red[3])) + 1);
}

// Symbol emission (dct_block.hpp:415-439) in three steps. count: one CTA per block, the cluster
// and category of every coefficient (its context depends only on the final neighbour levels) into
// the block's per-cluster symbol and raw-bit counts and the plane's category histogram.
__global__ void __launch_bounds__(256) fxv_enc_count(const int16_t* __restrict__ lev, EncBlk* __restrict__ blk,
                                                     const uint32_t* __restrict__ scan, EncHdr* __restrict__ eh) {
    __shared__ uint32_t cnt[kMaxCl + 1];
    __shared__ uint32_t cc[kMaxCl * kNCat];
    __shared__ uint8_t cmap[kRawCtx];
    const int b = blockIdx.x;
    const int64_t t = blockIdx.y;
    EncHdr& h = eh[t];
    if (!h.nonzero) return;
    for (int k = threadIdx.x; k < kMaxCl * kNCat; k += 256) cc[k] = 0;
    if (threadIdx.x <= kMaxCl) cnt[threadIdx.x] = 0;
    if (threadIdx.x < kRawCtx) cmap[threadIdx.x] = h.cmap[threadIdx.x];
    __syncthreads();
    const int16_t* L = lev + (t * 64 + b) * static_cast<int64_t>(kV);
    const uint32_t ns = blk[t * 64 + b].nsig;
    for (uint32_t pos = threadIdx.x; pos < ns; pos += 256) {
        const uint32_t e = scan[pos];
        const int i = e & 0xffff, fsum = (e >> 16) & 0xff, edge = e >> 24;
        const int cl = cmap[raw_ctx(fsum, nsum_lev(L, i, edge))];
        const int cat = bitw(static_cast<uint32_t>(abs(static_cast<int>(L[i]))));
        atomicAdd(&cnt[cl], 1u);
        if (cat) atomicAdd(&cnt[kMaxCl], static_cast<uint32_t>(cat));
        atomicAdd(&cc[cl * kNCat + cat], 1u);
    }
    __syncthreads();
    if (threadIdx.x <= kMaxCl) blk[t * 64 + b].cnt[threadIdx.x] = cnt[threadIdx.x];
    for (int k = threadIdx.x; k < kMaxCl * kNCat; k += 256)
        if (cc[k]) atomicAdd(&h.cc[k / kNCat][k % kNCat], cc[k]);
}

// prefix: one CTA per tile, the blocks' offsets within each plane and the bit stream, the plane
// lengths, and the zeroed bit-stream words.
__global__ void __launch_bounds__(64) fxv_enc_prefix(EncBlk* __restrict__ blk, EncHdr* __restrict__ eh,
                                                     uint8_t* __restrict__ work) {
    __shared__ uint32_t s_nbits;
    const int64_t t = blockIdx.x;
    EncHdr& h = eh[t];
    if (!h.nonzero) return;
    if (threadIdx.x <= kMaxCl) {
        const int k = threadIdx.x;
        uint32_t run = 0;
        for (int b = 0; b < 64; ++b) {
            blk[t * 64 + b].off[k] = run;
            run += blk[t * 64 + b].cnt[k];
        }
        if (k < kMaxCl) h.plane_n[k] = run;
        else {
            h.nbits = run;
            s_nbits = run;
        }
    }
    __syncthreads();
    uint32_t* W = reinterpret_cast<uint32_t*>(work + t * kWorkPerTile + kSymCap + kEncCap);
    const uint32_t nwords = (s_nbits + 31) / 32;
    for (uint32_t k = threadIdx.x; k < nwords; k += 64) W[k] = 0;
}

// write: one CTA per block; each thread takes 16 consecutive scan positions, a block-wide scan gives
// every position its rank within its cluster stream and its raw-bit offset, then symbols and bits
// go out (bits into u32 words by atomicOr, little-endian = the reference's LSB-first byte stream).
__global__ void __launch_bounds__(256) fxv_enc_write(const int16_t* __restrict__ lev, const EncBlk* __restrict__ blk,
                                                     const uint32_t* __restrict__ scan, const EncHdr* __restrict__ eh,
                                                     uint8_t* __restrict__ work) {
    __shared__ uint32_t sv[kMaxCl + 1][257];
    __shared__ uint32_t base[kMaxCl + 1];
    __shared__ uint8_t cmap[kRawCtx];
    const int b = blockIdx.x;
    const int64_t t = blockIdx.y;
    const EncHdr& h = eh[t];
    if (!h.nonzero) return;
    const int tid = threadIdx.x;
    if (tid < kRawCtx) cmap[tid] = h.cmap[tid];
    if (tid <= kMaxCl) {
        uint32_t pb = 0;
        if (tid < kMaxCl)
            for (int k = 0; k < tid; ++k) pb += h.plane_n[k];
        base[tid] = pb + blk[t * 64 + b].off[tid];
    }
    __syncthreads();
    const int16_t* L = lev + (t * 64 + b) * static_cast<int64_t>(kV);
    const uint32_t ns = blk[t * 64 + b].nsig;
    const uint32_t p0 = tid * 16, p1 = min(p0 + 16, ns);
    uint32_t c[kMaxCl + 1] = {};
    uint8_t cls[16], cats[16];
    for (uint32_t pos = p0; pos < p1; ++pos) {
        const uint32_t e = scan[pos];
        const int i = e & 0xffff, fsum = (e >> 16) & 0xff, edge = e >> 24;
        const int cl = cmap[raw_ctx(fsum, nsum_lev(L, i, edge))];
        const int cat = bitw(static_cast<uint32_t>(abs(static_cast<int>(L[i]))));
        cls[pos - p0] = static_cast<uint8_t>(cl);
        cats[pos - p0] = static_cast<uint8_t>(cat);
        ++c[cl];
        c[kMaxCl] += cat;
    }
#pragma unroll
    for (int k = 0; k <= kMaxCl; ++k) sv[k][tid] = c[k];
    __syncthreads();
    if (tid <= kMaxCl) {  // exclusive scan over the threads, one value per thread
        uint32_t run = 0;
        for (int k = 0; k < 256; ++k) {
            const uint32_t v = sv[tid][k];
            sv[tid][k] = run;
            run += v;
        }
    }
    __syncthreads();
    uint8_t* syms = work + t * kWorkPerTile;
    uint32_t* W = reinterpret_cast<uint32_t*>(work + t * kWorkPerTile + kSymCap + kEncCap);
    uint32_t k_cl[kMaxCl];
#pragma unroll
    for (int k = 0; k < kMaxCl; ++k) k_cl[k] = base[k] + sv[k][tid];
    uint32_t B = base[kMaxCl] + sv[kMaxCl][tid];
    auto put = [&](uint32_t v, int w) {
        if (w <= 0) return;
        const uint32_t wd = B >> 5, sh = B & 31;
        atomicOr(&W[wd], v << sh);
        if (sh + w > 32) atomicOr(&W[wd + 1], v >> (32 - sh));
        B += w;
    };
    for (uint32_t pos = p0; pos < p1; ++pos) {
        const int cl = cls[pos - p0], cat = cats[pos - p0];
        uint32_t kk = 0;
#pragma unroll
        for (int k = 0; k < kMaxCl; ++k)
            if (k == cl) kk = k_cl[k]++;
        syms[kk] = static_cast<uint8_t>(cat);
        if (cat > 0) {
            const int l = L[scan[pos] & 0xffff];
            const uint32_t a = static_cast<uint32_t>(abs(l));
            put(a - (1u << (cat - 1)), cat - 1);
            put(l < 0 ? 1u : 0u, 1);
        }
    }
}

// rANS encoding of one category plane (rans.hpp:83-131 model, 141-201 coder), one thread per plane.
__global__ void fxv_enc_rans(EncHdr* __restrict__ eh, uint8_t* __restrict__ work, int64_t n) {
    const int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    const int64_t t = g >> 3;
    const int cl = static_cast<int>(g & 7);
    if (t >= n) return;
    EncHdr& h = eh[t];
    if (!h.nonzero || cl >= h.K) return;
    const uint32_t pn = h.plane_n[cl];
    uint64_t sb = 0, eo = 0;
    for (int k = 0; k < cl; ++k) {
        sb += h.plane_n[k];
        eo += 2ull * h.plane_n[k] + 128;
    }
    h.enc_off[cl] = kSymCap + eo;
    h.enc_len[cl] = 0;
    if (pn == 0) return;
    const uint8_t* s = work + t * kWorkPerTile + sb;
    uint32_t counts[kNCat];
    for (int k = 0; k < kNCat; ++k) counts[k] = h.cc[cl][k];
    uint32_t freq[kNCat] = {}, cum[kNCat];
    uint32_t assigned = 0;
    int last = -1;
    for (int k = 0; k < kNCat; ++k) {
        if (!counts[k]) continue;
        uint32_t f = static_cast<uint32_t>((static_cast<uint64_t>(counts[k]) * kRansScale) / pn);
        if (f == 0) f = 1;
        freq[k] = f;
        assigned += f;
        last = k;
    }
    if (assigned > kRansScale && last >= 0) {
        uint32_t over = assigned - kRansScale;
        while (over > 0) {
            int big = -1;
            for (int k = 0; k < kNCat; ++k) {
                if (freq[k] <= 1) continue;
                if (big < 0 || freq[k] > freq[big]) big = k;
            }
            if (big < 0) break;
            --freq[big];
            --over;
        }
    } else if (assigned < kRansScale && last >= 0) {
        int big = 0;
        for (int k = 1; k < kNCat; ++k)
            if (freq[k] > freq[big]) big = k;
        freq[big] += kRansScale - assigned;
    }
    uint32_t cc = 0;
    uint64_t rcp[kNCat];  // floor(x / f) = umulhi64(x, ceil(2^64 / f)) for x < 2^32, f >= 2
    for (int k = 0; k < kNCat; ++k) {
        cum[k] = cc;
        cc += freq[k];
        h.freq[cl][k] = freq[k];
        rcp[k] = freq[k] > 1 ? (~0ull / freq[k]) + 1 : 0;
    }
    uint8_t* buf = work + t * kWorkPerTile + kSymCap + eo;
    const uint32_t cap = 2 * pn + 128;
    uint32_t ptr = cap;
    auto enc = [&](uint32_t& x, uint8_t sym) {
        const uint32_t f = freq[sym], c = cum[sym];
        const uint32_t xmax = ((kRansL >> 12) << 8) * f;
        while (x >= xmax) {
            buf[--ptr] = static_cast<uint8_t>(x & 0xffu);
            x >>= 8;
        }
        const uint32_t qt = f > 1 ? static_cast<uint32_t>(__umul64hi(x, rcp[sym])) : x;
        x = (qt << 12) + (x - qt * f) + c;
    };
    auto put4 = [&](uint32_t x) {
        ptr -= 4;
        buf[ptr] = static_cast<uint8_t>(x);
        buf[ptr + 1] = static_cast<uint8_t>(x >> 8);
        buf[ptr + 2] = static_cast<uint8_t>(x >> 16);
        buf[ptr + 3] = static_cast<uint8_t>(x >> 24);
    };
    if (pn < 4096) {
        uint32_t x0 = kRansL;
        for (uint32_t i = pn; i-- > 0;) enc(x0, s[i]);
        put4(x0);
    } else {
        uint32_t x0 = kRansL, x1 = kRansL, x2 = kRansL, x3 = kRansL;
        const int64_t sn = pn, ng = sn / 4, base = ng * 4;
        for (int64_t i = sn - 1; i >= base; --i) {
            uint32_t& x = (i & 3) == 0 ? x0 : (i & 3) == 1 ? x1 : (i & 3) == 2 ? x2 : x3;
            enc(x, s[i]);
        }
        for (int64_t gg = ng - 1; gg >= 0; --gg) {
            enc(x3, s[4 * gg + 3]);
            enc(x2, s[4 * gg + 2]);
            enc(x1, s[4 * gg + 1]);
            enc(x0, s[4 * gg]);
        }
        put4(x3);
        put4(x2);
        put4(x1);
        put4(x0);
    }
    h.enc_start[cl] = ptr;
    h.enc_len[cl] = cap - ptr;
}

__device__ __forceinline__ void hput_var(uint8_t* o, int& n, uint32_t v) {
    while (v >= 0x80) {
        o[n++] = static_cast<uint8_t>(v | 0x80u);
        v >>= 7;
    }
    o[n++] = static_cast<uint8_t>(v);
}

// Payload assembly (dct_block.hpp:441-483), one warp per tile: lane 0 writes the headers to shared
// memory, the warp copies headers, rANS streams and raw bits into the compact output.
__global__ void __launch_bounds__(32) fxv_enc_assemble(const EncBlk* __restrict__ blk, const EncHdr* __restrict__ eh,
                                                       const uint8_t* __restrict__ work, uint8_t* __restrict__ out,
                                                       unsigned long long* __restrict__ out_ctr, uint64_t out_cap,
                                                       EncOut* __restrict__ res, int dc_predict) {
    __shared__ uint8_t hb[2048];
    __shared__ int hend[kMaxCl + 1];
    __shared__ int s_hlen;
    __shared__ unsigned long long s_off;
    __shared__ uint32_t s_total;
    const int64_t t = blockIdx.x;
    const EncHdr& h = eh[t];
    const int lane = threadIdx.x;
    if (!h.nonzero) {
        if (lane == 0) res[t] = EncOut{0, 0, 0};
        return;
    }
    const int K = h.K;
    const uint32_t nbytes = (h.nbits + 7) / 8;
    if (lane == 0) {
        int n = 0;
        int32_t dcl[64];
        uint32_t ns[64];
        for (int b = 0; b < 64; ++b) {
            dcl[b] = blk[t * 64 + b].dclev;
            ns[b] = blk[t * 64 + b].nsig;
        }
        for (int b = 0; b < 64; ++b) {
            const int32_t pred = dc_predict ? causal_pred(dcl, b) : 0;
            const int32_t r = dcl[b] - pred;
            hput_var(hb, n, (static_cast<uint32_t>(r) << 1) ^ static_cast<uint32_t>(r >> 31));
        }
        for (int b = 0; b < 64; ++b) {
            const int32_t pred = dc_predict ? causal_pred(ns, b) : 0;
            const int32_t r = static_cast<int32_t>(ns[b]) - pred;
            hput_var(hb, n, (static_cast<uint32_t>(r) << 1) ^ static_cast<uint32_t>(r >> 31));
        }
        hb[n++] = static_cast<uint8_t>(K);
        for (int r = 0; r < kRawCtx; ++r) hb[n++] = h.cmap[r];
        uint32_t total = 0;
        for (int cl = 0; cl < K; ++cl) {
            const uint32_t pn = h.plane_n[cl];
            hput_var(hb, n, pn);
            if (pn) {
                hput_var(hb, n, h.enc_len[cl]);
                uint32_t nused = 0;
                for (int k = 0; k < kNCat; ++k) nused += h.freq[cl][k] != 0;
                hput_var(hb, n, nused);
                for (int k = 0; k < kNCat; ++k)
                    if (h.freq[cl][k]) {
                        hb[n++] = static_cast<uint8_t>(k);
                        hput_var(hb, n, h.freq[cl][k]);
                    }
                total += h.enc_len[cl];
            }
            hend[cl] = n;
        }
        hput_var(hb, n, nbytes);
        s_hlen = n;
        total += static_cast<uint32_t>(n) + nbytes;
        s_total = total;
        const unsigned long long off = atomicAdd(out_ctr, static_cast<unsigned long long>(total));
        s_off = off;
        res[t] = EncOut{off, total, off + total > out_cap ? 1u : 0u};
    }
    __syncwarp();
    if (s_off + s_total > out_cap) return;
    uint8_t* o = out + s_off;
    const uint8_t* wt = work + t * kWorkPerTile;
    int hpos = 0;
    uint64_t op = 0;
    for (int cl = 0; cl <= K; ++cl) {
        const int he = cl < K ? hend[cl] : s_hlen;
        for (int k = lane; k < he - hpos; k += 32) o[op + k] = hb[hpos + k];
        op += he - hpos;
        hpos = he;
        if (cl < K && h.plane_n[cl]) {
            const uint8_t* src = wt + h.enc_off[cl] + h.enc_start[cl];
            const uint32_t L = h.enc_len[cl];
            for (uint32_t k = lane; k < L; k += 32) o[op + k] = src[k];
            op += L;
        }
    }
    const uint8_t* bits = wt + kSymCap + kEncCap;
    for (uint32_t k = lane; k < nbytes; k += 32) o[op + k] = bits[k];
}

}  // namespace
}  // namespace fxk

namespace fxh {

using namespace fxk;

namespace {
CodecStatus cerr(const char* what, cudaError_t e) {
    return {8, std::string(what) + ": " + cudaGetErrorString(e)};
}
constexpr int kMaxEncBatch = 296;
constexpr int kMaxReconBatch = 296;
constexpr int64_t kMaxDecBatch = 8192;
}  // namespace

FxvCodec::~FxvCodec() {
    for (void* p : {scan_, hdr_, syms_, ent_, recon_, ctr_, elev_, ecoef_, eblk_, ehdr_, ework_, eout_, eres_, htiles_})
        if (p) cudaFree(p);
    if (pinned_) cudaFreeHost(pinned_);
}

void* FxvCodec::grow(void*& p, size_t& cap, size_t want) {
    if (want <= cap && p) return p;
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
    if (cudaMalloc(&p, want) != cudaSuccess) {
        p = nullptr;
        return nullptr;
    }
    cap = want;
    return p;
}

CodecStatus FxvCodec::tables(cudaStream_t s) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (scan_ && dev == dev_) return {};
    if (scan_) cudaFree(scan_);
    scan_ = nullptr;
    dev_ = dev;
    // frequency-ascending scan, stable within a shell (dct_block.hpp:67-86), and its inverse
    std::vector<uint32_t> scan(kV);
    std::vector<uint16_t> rank(kV + 48);  // then the first scan position of each shell f = 0..46
    int pos = 0;
    for (int f = 0; f <= 45; ++f) {
        rank[kV + f] = static_cast<uint16_t>(pos);
        for (int i = 0; i < kV; ++i) {
            const int z = i >> 8, y = (i >> 4) & 15, x = i & 15;
            if (z + y + x != f) continue;
            const uint32_t edge = (z > 0 ? 1u : 0u) | (y > 0 ? 2u : 0u) | (x > 0 ? 4u : 0u);
            scan[pos] = static_cast<uint32_t>(i) | (static_cast<uint32_t>(f) << 16) | (edge << 24);
            rank[i] = static_cast<uint16_t>(pos);
            ++pos;
        }
    }
    rank[kV + 46] = rank[kV + 47] = static_cast<uint16_t>(kV);
    if (cudaMalloc(&scan_, kV * 6 + 96) != cudaSuccess) return {8, "cudaMalloc: codec tables"};
    cudaMemcpyAsync(scan_, scan.data(), kV * 4, cudaMemcpyHostToDevice, s);
    cudaMemcpyAsync(static_cast<uint8_t*>(scan_) + kV * 4, rank.data(), (kV + 48) * 2, cudaMemcpyHostToDevice, s);
    const cudaError_t e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? CodecStatus{} : cerr("codec tables", e);
}

CodecStatus FxvCodec::decode(const uint8_t* d_blob, const FxvDecTile* tiles, int64_t n, const FxvParams& p,
                             uint8_t* d_out, int64_t dz, int64_t dy, int64_t dx, float* d_recon, cudaStream_t s) {
    launches_ = 0;
    if (n <= 0) return {};
    if (CodecStatus st = tables(s); st.code) return st;
    const uint32_t* scan = static_cast<const uint32_t*>(scan_);
    cudaFuncSetAttribute(fxv_dec_walk, cudaFuncAttributeMaxDynamicSharedMemorySize, (kV + kWalkTiles * 257) * 4);
    for (int64_t t0 = 0; t0 < n; t0 += kMaxDecBatch) {
        const int64_t nb = std::min<int64_t>(kMaxDecBatch, n - t0);
        if (!grow(htiles_, htiles_cap_, sizeof(FxvDecTile) * nb) || !grow(hdr_, hdr_cap_, sizeof(DecHdr) * nb) ||
            !grow(ctr_, ctr_cap_, 64))
            return {8, "cudaMalloc: decode scratch"};
        cudaMemcpyAsync(htiles_, tiles + t0, sizeof(FxvDecTile) * nb, cudaMemcpyHostToDevice, s);
        size_t sym_want = std::max<size_t>(syms_cap_, 16u << 20), ent_want = std::max<size_t>(ent_cap_, 16u << 20);
        for (int attempt = 0; attempt < 2; ++attempt) {
            if (!grow(syms_, syms_cap_, sym_want) || !grow(ent_, ent_cap_, ent_want))
                return {8, "cudaMalloc: decode scratch"};
            cudaMemsetAsync(ctr_, 0, 16, s);
            fxv_dec_parse<<<static_cast<unsigned>((nb + 127) / 128), 128, 0, s>>>(
                d_blob, static_cast<const FxvDecTile*>(htiles_), nb, p.dc_predict, static_cast<DecHdr*>(hdr_),
                static_cast<unsigned long long*>(ctr_), syms_cap_, ent_cap_ / sizeof(float2));
            ++launches_;
            unsigned long long need[2] = {0, 0};
            cudaMemcpyAsync(need, ctr_, 16, cudaMemcpyDeviceToHost, s);
            if (cudaError_t e = cudaStreamSynchronize(s); e != cudaSuccess) return cerr("fxv_dec_parse", e);
            if (need[0] <= syms_cap_ && need[1] * sizeof(float2) <= ent_cap_) break;
            sym_want = std::max<size_t>(sym_want, need[0]);
            ent_want = std::max<size_t>(ent_want, need[1] * sizeof(float2));
        }
        fxv_dec_rans<<<static_cast<unsigned>(nb), 256, 0, s>>>(d_blob, static_cast<DecHdr*>(hdr_),
                                                                static_cast<uint8_t*>(syms_));
        // one serial walker per tile: few tiles per CTA so that small batches still spread over the SMs
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev_);
        const int tpc = static_cast<int>(std::min<int64_t>(kWalkTiles, std::max<int64_t>(1, (nb + 4 * sms - 1) / (4 * sms))));
        fxv_dec_walk<<<static_cast<unsigned>((nb + tpc - 1) / tpc), tpc, (kV + tpc * 257) * 4, s>>>(
            d_blob, static_cast<DecHdr*>(hdr_), static_cast<const uint8_t*>(syms_), scan, p,
            static_cast<float2*>(ent_), nb);
        launches_ += 2;
        for (int64_t r0 = 0; r0 < nb; r0 += kMaxReconBatch) {
            const int64_t nr = std::min<int64_t>(kMaxReconBatch, nb - r0);
            float* rec = d_recon ? d_recon + (t0 + r0) * static_cast<int64_t>(kTileV)
                                 : static_cast<float*>(grow(recon_, recon_cap_, sizeof(float) * kTileV * kMaxReconBatch));
            if (!rec) return {8, "cudaMalloc: decode reconstruction"};
            fxv_dec_recon<<<static_cast<unsigned>(nr), 512, 0, s>>>(
                static_cast<const DecHdr*>(hdr_), static_cast<const float2*>(ent_), p, rec, r0,
                static_cast<const FxvDecTile*>(htiles_), d_out, dz, dy, dx);
            ++launches_;
        }
        std::vector<int32_t> errs(static_cast<size_t>(nb));
        cudaMemcpy2DAsync(errs.data(), sizeof(int32_t), hdr_, sizeof(DecHdr), sizeof(int32_t), static_cast<size_t>(nb),
                          cudaMemcpyDeviceToHost, s);
        if (cudaError_t e = cudaStreamSynchronize(s); e != cudaSuccess) return cerr("fxv decode", e);
        for (int64_t k = 0; k < nb; ++k)
            if (errs[static_cast<size_t>(k)]) {
                static const char* what[] = {"", "truncated field", "field out of range", "category stream underrun",
                                             "scratch exhausted"};
                const int c = errs[static_cast<size_t>(k)];
                return {c == E_SCRATCH ? 8 : 5, std::string("fxvol tile ") + std::to_string(t0 + k) + ": " +
                                                    (c >= 1 && c <= 4 ? what[c] : "decode error")};
            }
    }
    return {};
}

CodecStatus FxvCodec::encode(const uint8_t* src8, const float* src32, int64_t dz, int64_t dy, int64_t dx,
                             const FxvEncTile* tiles, int64_t n, const FxvParams& p, std::vector<uint8_t>& payload,
                             std::vector<uint64_t>& offsets, std::vector<uint32_t>& lengths, cudaStream_t s,
                       bool zero_slots) {
    launches_ = 0;
    if (n <= 0) return {};
    if (CodecStatus st = tables(s); st.code) return st;
    const uint32_t* scan = static_cast<const uint32_t*>(scan_);
    const uint16_t* rank = reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(scan_) + kV * 4);
    const uint16_t* shell = rank + kV;
    const int64_t B = std::min<int64_t>(kMaxEncBatch, n);
    if (!grow(elev_, elev_cap_, sizeof(int16_t) * kV * 64 * B) || !grow(ecoef_, ecoef_cap_, sizeof(float) * kV * 64 * B) ||
        !grow(eblk_, eblk_cap_, sizeof(EncBlk) * 64 * B) || !grow(ehdr_, ehdr_cap_, sizeof(EncHdr) * B) ||
        !grow(ework_, ework_cap_, kWorkPerTile * B) || !grow(htiles_, htiles_cap_, sizeof(FxvEncTile) * B) ||
        !grow(ctr_, ctr_cap_, 64))
        return {8, "cudaMalloc: encode scratch"};
    // compact output: sized for typical payloads, grown (and the assembly re-run) when exceeded
    size_t out_want = std::max<size_t>(eout_cap_, static_cast<size_t>(B) * (256u << 10));
    if (!grow(eres_, eres_cap_, sizeof(EncOut) * B)) return {8, "cudaMalloc: encode scratch"};
    std::vector<EncOut> res(static_cast<size_t>(B));
    EncHdr* eh = static_cast<EncHdr*>(ehdr_);
    int16_t* lev = static_cast<int16_t*>(elev_);
    float* coef = static_cast<float*>(ecoef_);
    EncBlk* blk = static_cast<EncBlk*>(eblk_);
    uint8_t* work = static_cast<uint8_t*>(ework_);
    EncOut* dres = static_cast<EncOut*>(eres_);
    for (int64_t t0 = 0; t0 < n; t0 += B) {
        const int64_t nb = std::min<int64_t>(B, n - t0);
        cudaMemcpyAsync(htiles_, tiles + t0, sizeof(FxvEncTile) * nb, cudaMemcpyHostToDevice, s);
        cudaMemsetAsync(ehdr_, 0, sizeof(EncHdr) * nb, s);
        const dim3 gq(64, static_cast<unsigned>(nb));
        if (src32)
            fxv_enc_quant<true><<<gq, 256, 0, s>>>(nullptr, src32, dz, dy, dx, static_cast<const FxvEncTile*>(htiles_),
                                                   p, rank, lev, coef, blk, eh, zero_slots ? 0 : 1);
        else
            fxv_enc_quant<false><<<gq, 256, 0, s>>>(src8, nullptr, dz, dy, dx, static_cast<const FxvEncTile*>(htiles_),
                                                    p, rank, lev, coef, blk, eh, zero_slots ? 0 : 1);
        fxv_enc_hist<<<gq, 256, 0, s>>>(lev, blk, scan, eh);
        fxv_enc_cluster<<<static_cast<unsigned>(nb), 32, 0, s>>>(eh);
        launches_ += 3;
        if (p.rdoq) {
            fxv_enc_rdoq<<<gq, 128, 0, s>>>(lev, coef, blk, scan, shell, eh, p);
            ++launches_;
        }
        fxv_enc_count<<<gq, 256, 0, s>>>(lev, blk, scan, eh);
        fxv_enc_prefix<<<static_cast<unsigned>(nb), 64, 0, s>>>(blk, eh, work);
        fxv_enc_write<<<gq, 256, 0, s>>>(lev, blk, scan, eh, work);
        fxv_enc_rans<<<static_cast<unsigned>((nb * 8 + 127) / 128), 128, 0, s>>>(eh, work, nb);
        launches_ += 4;
        unsigned long long used = 0;
        for (int attempt = 0; attempt < 2; ++attempt) {
            if (!grow(eout_, eout_cap_, out_want)) return {8, "cudaMalloc: encode output"};
            cudaMemsetAsync(ctr_, 0, 8, s);
            fxv_enc_assemble<<<static_cast<unsigned>(nb), 32, 0, s>>>(
                blk, eh, work, static_cast<uint8_t*>(eout_), static_cast<unsigned long long*>(ctr_), eout_cap_, dres,
                p.dc_predict);
            ++launches_;
            cudaMemcpyAsync(&used, ctr_, 8, cudaMemcpyDeviceToHost, s);
            if (cudaError_t e = cudaStreamSynchronize(s); e != cudaSuccess) return cerr("fxv encode", e);
            if (used <= eout_cap_) break;
            out_want = static_cast<size_t>(used);
        }
        if (used > eout_cap_) return {8, "fxvol encode: output buffer exhausted"};
        cudaMemcpyAsync(res.data(), dres, sizeof(EncOut) * nb, cudaMemcpyDeviceToHost, s);
        if (used > pinned_cap_) {
            if (pinned_) cudaFreeHost(pinned_);
            pinned_ = nullptr;
            pinned_cap_ = 0;
            if (cudaMallocHost(&pinned_, used) != cudaSuccess) return {8, "cudaMallocHost: encode staging"};
            pinned_cap_ = used;
        }
        if (used) cudaMemcpyAsync(pinned_, eout_, used, cudaMemcpyDeviceToHost, s);
        if (cudaError_t e = cudaStreamSynchronize(s); e != cudaSuccess) return cerr("fxv encode", e);
        const uint64_t base = payload.size();
        payload.insert(payload.end(), static_cast<uint8_t*>(pinned_), static_cast<uint8_t*>(pinned_) + used);
        for (int64_t k = 0; k < nb; ++k) {
            const EncOut& r = res[static_cast<size_t>(k)];
            offsets.push_back(base + r.off);
            lengths.push_back(r.len);
        }
    }
    return {};
}

}  // namespace fxh
