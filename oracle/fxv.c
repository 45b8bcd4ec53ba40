/* fxv.c — CPU oracle for the .fxvol chunk codec. TEST INFRASTRUCTURE ONLY (see fxv.h). */
#include "fxv.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

enum { N = 16, H = 8, V = 4096, SIDE = 64, BPA = 4, NBLK = 64 };
enum { MAG_CAP = 3, SUM_B = 6, BAND_B = 4, RAW_CTX = 24, MAX_CL = 8, NCAT = 18 };
#define RANS_L (1u << 23)
#define RANS_BITS 12u
#define RANS_SCALE (1u << 12)
#define INTERLEAVE_MIN 4096u

/* error codes (the reference's Errc::decode_error cases, grouped) */
enum { E_TRUNC = -1, E_RANGE = -2, E_UNDERRUN = -3, E_NOMEM = -4 };

/* ---- DCT-16 (dct.hpp:27-53 basis; transform order of the oracle's scalar shim) ---- */
/* The DCT-16 half bases: the reference's formula (dct.hpp:43 — f32 argument pi (2n+1) k / 32, f32
 * c_k) with the cosine correctly rounded, written out so every build uses the same values (libm's
 * cosf and a compiler's compile-time evaluation disagree by an ulp at one argument). */
static const float g_me[H][H] = {
    {0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f, 0x1p-2f},
    {0x1.63150ap-2f, 0x1.2d062ep-2f, 0x1.92469ap-3f, 0x1.1a8556p-4f, -0x1.1a855ep-4f, -0x1.9246a2p-3f, -0x1.2d063p-2f, -0x1.63150cp-2f},
    {0x1.4e7ae8p-2f, 0x1.1517a8p-3f, -0x1.1517acp-3f, -0x1.4e7aeap-2f, -0x1.4e7ae8p-2f, -0x1.151798p-3f, 0x1.1517bp-3f, 0x1.4e7aeap-2f},
    {0x1.2d062ep-2f, -0x1.1a855ep-4f, -0x1.63150cp-2f, -0x1.92469p-3f, 0x1.924694p-3f, 0x1.63150ap-2f, 0x1.1a8546p-4f, -0x1.2d0632p-2f},
    {0x1.fffffep-3f, -0x1.fffffep-3f, -0x1.fffffap-3f, 0x1.000006p-2f, 0x1.fffffep-3f, -0x1.00000ap-2f, -0x1.fffff4p-3f, 0x1p-2f},
    {0x1.92469ap-3f, -0x1.63150cp-2f, 0x1.1a8566p-4f, 0x1.2d0628p-2f, -0x1.2d0632p-2f, -0x1.1a84fap-4f, 0x1.63150cp-2f, -0x1.924694p-3f},
    {0x1.1517a8p-3f, -0x1.4e7ae8p-2f, 0x1.4e7aeep-2f, -0x1.1517bep-3f, -0x1.1517bap-3f, 0x1.4e7ae4p-2f, -0x1.4e7aeep-2f, 0x1.1517bep-3f},
    {0x1.1a8556p-4f, -0x1.92469p-3f, 0x1.2d0628p-2f, -0x1.631508p-2f, 0x1.63150ap-2f, -0x1.2d063ap-2f, 0x1.9246c6p-3f, -0x1.1a852p-4f},
};
static const float g_mo[H][H] = {
    {0x1.684b9cp-2f, 0x1.5a730cp-2f, 0x1.3f4a22p-2f, 0x1.17dc14p-2f, 0x1.cb598cp-3f, 0x1.5553ep-3f, 0x1.a46086p-4f, 0x1.1be35p-5f},
    {0x1.5a730cp-2f, 0x1.cb598cp-3f, 0x1.1be33ap-5f, -0x1.5553e8p-3f, -0x1.3f4a22p-2f, -0x1.684b9cp-2f, -0x1.17dc12p-2f, -0x1.a4607ep-4f},
    {0x1.3f4a22p-2f, 0x1.1be35p-5f, -0x1.17dc14p-2f, -0x1.5a730cp-2f, -0x1.a4607ep-4f, 0x1.cb59ap-3f, 0x1.684b9cp-2f, 0x1.5553e8p-3f},
    {0x1.17dc14p-2f, -0x1.5553e8p-3f, -0x1.5a730cp-2f, 0x1.1be388p-5f, 0x1.684b9cp-2f, 0x1.a46062p-4f, -0x1.3f4a2ap-2f, -0x1.cb5998p-3f},
    {0x1.cb598cp-3f, -0x1.3f4a22p-2f, -0x1.a4607ep-4f, 0x1.684b9ep-2f, -0x1.1be36ap-5f, -0x1.5a7306p-2f, 0x1.5553eap-3f, 0x1.17dc0ep-2f},
    {0x1.5553ep-3f, -0x1.684b9cp-2f, 0x1.cb598ep-3f, 0x1.a46062p-4f, -0x1.5a730cp-2f, 0x1.17dc26p-2f, 0x1.1be2ccp-5f, -0x1.3f4a2p-2f},
    {0x1.a46086p-4f, -0x1.17dc16p-2f, 0x1.684b9ap-2f, -0x1.3f4a2ap-2f, 0x1.5553eap-3f, 0x1.1be2ccp-5f, -0x1.cb595ep-3f, 0x1.5a7306p-2f},
    {0x1.1be35p-5f, -0x1.a4607ep-4f, 0x1.5553d4p-3f, -0x1.cb5976p-3f, 0x1.17dc0ep-2f, -0x1.3f4a0cp-2f, 0x1.5a7306p-2f, -0x1.684b9ep-2f},
};
typedef struct {
    uint16_t idx;
    uint8_t fsum, edge;
} scan_e;
static scan_e g_scan[V];
static int g_ready;

static void init_tables(void) {
    if (g_ready) return;
    /* frequency-ascending scan, stable within a shell (dct_block.hpp:67-86) */
    int pos = 0;
    for (int f = 0; f <= 3 * (N - 1); ++f)
        for (int i = 0; i < V; ++i) {
            const int z = i / (N * N), y = (i / N) % N, x = i % N;
            if (z + y + x != f) continue;
            g_scan[pos].idx = (uint16_t)i;
            g_scan[pos].fsum = (uint8_t)f;
            g_scan[pos].edge = (uint8_t)((z > 0 ? 1 : 0) | (y > 0 ? 2 : 0) | (x > 0 ? 4 : 0));
            ++pos;
        }
    g_ready = 1;
}

static void dct1_fwd(const float* x, float* X) {
    float s[H], d[H];
    for (int n = 0; n < H; ++n) {
        s[n] = x[n] + x[N - 1 - n];
        d[n] = x[n] - x[N - 1 - n];
    }
    for (int k = 0; k < H; ++k) {
        float e = 0.0f, o = 0.0f;
        for (int n = 0; n < H; ++n) {
            const float pe = g_me[k][n] * s[n], po = g_mo[k][n] * d[n];
            e = e + pe;
            o = o + po;
        }
        X[2 * k] = e;
        X[2 * k + 1] = o;
    }
}

static void dct1_inv(const float* X, float* x) {
    float E[H], O[H];
    for (int n = 0; n < H; ++n) E[n] = O[n] = 0.0f;
    for (int k = 0; k < H; ++k)
        for (int n = 0; n < H; ++n) {
            const float pe = g_me[k][n] * X[2 * k], po = g_mo[k][n] * X[2 * k + 1];
            E[n] = E[n] + pe;
            O[n] = O[n] + po;
        }
    for (int n = 0; n < H; ++n) {
        x[n] = E[n] + O[n];
        x[N - 1 - n] = E[n] - O[n];
    }
}

static void dct3(float* d, void (*one)(const float*, float*)) {
    float in[N], out[N];
    for (int z = 0; z < N; ++z)
        for (int y = 0; y < N; ++y) {
            float* p = d + (z * N + y) * N;
            for (int i = 0; i < N; ++i) in[i] = p[i];
            one(in, out);
            for (int i = 0; i < N; ++i) p[i] = out[i];
        }
    for (int z = 0; z < N; ++z)
        for (int x = 0; x < N; ++x) {
            float* p = d + z * N * N + x;
            for (int i = 0; i < N; ++i) in[i] = p[i * N];
            one(in, out);
            for (int i = 0; i < N; ++i) p[i * N] = out[i];
        }
    for (int y = 0; y < N; ++y)
        for (int x = 0; x < N; ++x) {
            float* p = d + y * N + x;
            for (int i = 0; i < N; ++i) in[i] = p[i * N * N];
            one(in, out);
            for (int i = 0; i < N; ++i) p[i * N * N] = out[i];
        }
}

void fxv_dct3_fwd(float* blk) {
    init_tables();
    dct3(blk, dct1_fwd);
}
void fxv_dct3_inv(float* blk) {
    init_tables();
    dct3(blk, dct1_inv);
}

void fxv_params_default(fxv_params* p, float q) {
    p->q = q;
    p->hf_exp = 0.65f;
    p->dz_frac = 0.80f;
    p->rdoq = 1;
    p->rdoq_lambda = 0.15f;
    p->deblock = 1;
    p->deblock_beta = 2.5f;
    p->deblock_tc = 0.5f;
    p->dc_predict = 1;
}

/* dct_block.hpp:91-94 */
static void step_table(const fxv_params* p, float* stepv) {
    for (int f = 0; f < 3 * N; ++f) stepv[f] = p->q * powf(1.0f + (float)f, p->hf_exp);
}

/* ---- byte buffer + LEB128 varints (entropy.hpp:35-77) ---- */
typedef struct {
    uint8_t* b;
    size_t n, cap;
    int oom;
} buf_t;

static void buf_push(buf_t* o, uint8_t v) {
    if (o->n == o->cap) {
        size_t nc = o->cap ? o->cap * 2 : 4096;
        uint8_t* nb = (uint8_t*)realloc(o->b, nc);
        if (!nb) {
            o->oom = 1;
            return;
        }
        o->b = nb;
        o->cap = nc;
    }
    o->b[o->n++] = v;
}

static void buf_append(buf_t* o, const uint8_t* p, size_t n) {
    for (size_t i = 0; i < n; ++i) buf_push(o, p[i]);
}

static void put_var(buf_t* o, uint32_t v) {
    while (v >= 0x80) {
        buf_push(o, (uint8_t)(v | 0x80u));
        v >>= 7;
    }
    buf_push(o, (uint8_t)v);
}

static int get_var(const uint8_t* b, size_t n, size_t* p, uint32_t* out) {
    uint32_t v = 0;
    int sh = 0;
    uint8_t byte;
    do {
        if (*p >= n) return E_TRUNC;
        if (sh >= 32) return E_RANGE;
        byte = b[(*p)++];
        v |= (uint32_t)(byte & 0x7fu) << sh;
        sh += 7;
    } while (byte & 0x80u);
    *out = v;
    return 0;
}

/* ---- rANS (rans.hpp:22-279) ---- */
typedef struct {
    uint16_t freq[256], cum[256];
    uint8_t slot[RANS_SCALE];
} model_t;

static void model_cum(model_t* m) {
    uint32_t c = 0;
    for (int s = 0; s < 256; ++s) {
        m->cum[s] = (uint16_t)c;
        for (uint32_t i = 0; i < m->freq[s]; ++i) m->slot[c + i] = (uint8_t)s;
        c += m->freq[s];
    }
}

/* RansModel::from_counts (rans.hpp:83-131) */
static void model_from_counts(model_t* m, const uint64_t* counts) {
    memset(m, 0, sizeof *m);
    uint64_t total = 0;
    for (int s = 0; s < 256; ++s) total += counts[s];
    if (total == 0) {
        for (int s = 0; s < 256; ++s) m->freq[s] = (uint16_t)(RANS_SCALE / 256);
    } else {
        uint32_t assigned = 0;
        int last = -1;
        for (int s = 0; s < 256; ++s) {
            if (counts[s] == 0) continue;
            uint32_t f = (uint32_t)((counts[s] * RANS_SCALE) / total);
            if (f == 0) f = 1;
            m->freq[s] = (uint16_t)f;
            assigned += f;
            last = s;
        }
        if (assigned > RANS_SCALE && last >= 0) {
            uint32_t over = assigned - RANS_SCALE;
            while (over > 0) {
                int big = -1;
                for (int s = 0; s < 256; ++s) {
                    if (m->freq[s] <= 1) continue;
                    if (big < 0 || m->freq[s] > m->freq[big]) big = s;
                }
                if (big < 0) break;
                --m->freq[big];
                --over;
            }
        } else if (assigned < RANS_SCALE && last >= 0) {
            int big = 0;
            for (int s = 1; s < 256; ++s)
                if (m->freq[s] > m->freq[big]) big = s;
            m->freq[big] = (uint16_t)(m->freq[big] + (RANS_SCALE - assigned));
        }
    }
    model_cum(m);
}

/* rans_encode (rans.hpp:141-201): returns the stream in *out (malloc'd) */
static size_t rans_encode(const uint8_t* data, size_t n, const model_t* m, uint8_t** out) {
    const size_t cap = n * 2 + 128;
    uint8_t* buf = (uint8_t*)malloc(cap);
    size_t ptr = cap;
#define ENC(x, s)                                                                \
    do {                                                                         \
        const uint32_t f_ = m->freq[(s)], c_ = m->cum[(s)];                      \
        const uint32_t xmax_ = ((RANS_L >> RANS_BITS) << 8) * f_;                \
        while ((x) >= xmax_) {                                                   \
            buf[--ptr] = (uint8_t)((x)&0xffu);                                   \
            (x) >>= 8;                                                           \
        }                                                                        \
        (x) = (((x) / f_) << RANS_BITS) + ((x) % f_) + c_;                       \
    } while (0)
    if (n < INTERLEAVE_MIN) {
        uint32_t x0 = RANS_L;
        for (size_t i = n; i-- > 0;) ENC(x0, data[i]);
        ptr -= 4;
        memcpy(buf + ptr, &x0, 4);
    } else {
        uint32_t x0 = RANS_L, x1 = RANS_L, x2 = RANS_L, x3 = RANS_L;
        const int64_t sn = (int64_t)n, ng = sn / 4, base = ng * 4;
        for (int64_t i = sn - 1; i >= base; --i) switch (i & 3) {
            case 0: ENC(x0, data[i]); break;
            case 1: ENC(x1, data[i]); break;
            case 2: ENC(x2, data[i]); break;
            default: ENC(x3, data[i]); break;
            }
        for (int64_t g = ng - 1; g >= 0; --g) {
            const size_t b = (size_t)(4 * g);
            ENC(x3, data[b + 3]);
            ENC(x2, data[b + 2]);
            ENC(x1, data[b + 1]);
            ENC(x0, data[b]);
        }
        ptr -= 4;
        memcpy(buf + ptr, &x3, 4);
        ptr -= 4;
        memcpy(buf + ptr, &x2, 4);
        ptr -= 4;
        memcpy(buf + ptr, &x1, 4);
        ptr -= 4;
        memcpy(buf + ptr, &x0, 4);
    }
#undef ENC
    const size_t len = cap - ptr;
    memmove(buf, buf + ptr, len);
    *out = buf;
    return len;
}

/* rans_decode (rans.hpp:204-277) */
static void rans_decode(const uint8_t* st, size_t len, size_t n, const model_t* m, uint8_t* out) {
    memset(out, 0, n);
    if (len == 0) return;
    size_t p = 0;
    const int K = n >= INTERLEAVE_MIN ? 4 : 1;
    const uint32_t mask = RANS_SCALE - 1;
#define RD4(v)                           \
    do {                                 \
        (v) = RANS_L;                    \
        if (p + 4 <= len) {              \
            memcpy(&(v), st + p, 4);     \
            p += 4;                      \
        }                                \
    } while (0)
#define DEC(x, dst)                                                              \
    do {                                                                         \
        const uint32_t s_ = m->slot[(x)&mask];                                   \
        (x) = (uint32_t)m->freq[s_] * ((x) >> RANS_BITS) + ((x)&mask) - m->cum[s_]; \
        while ((x) < RANS_L && p < len) (x) = ((x) << 8) | st[p++];              \
        (dst) = (uint8_t)s_;                                                     \
    } while (0)
    if (K == 1) {
        uint32_t x0;
        RD4(x0);
        for (size_t i = 0; i < n; ++i) DEC(x0, out[i]);
    } else {
        uint32_t x0, x1, x2, x3;
        RD4(x0);
        RD4(x1);
        RD4(x2);
        RD4(x3);
        const int64_t sn = (int64_t)n, ng = sn / 4, base = ng * 4;
        for (int64_t g = 0; g < ng; ++g) {
            const size_t b = (size_t)(4 * g);
            DEC(x0, out[b]);
            DEC(x1, out[b + 1]);
            DEC(x2, out[b + 2]);
            DEC(x3, out[b + 3]);
        }
        for (int64_t i = base; i < sn; ++i) switch (i & 3) {
            case 0: DEC(x0, out[i]); break;
            case 1: DEC(x1, out[i]); break;
            case 2: DEC(x2, out[i]); break;
            default: DEC(x3, out[i]); break;
            }
    }
#undef RD4
#undef DEC
}

/* encode_plane (entropy.hpp:82-108) */
static void encode_plane(buf_t* o, const uint8_t* plane, size_t n) {
    put_var(o, (uint32_t)n);
    if (n == 0) return;
    uint64_t counts[256] = {0};
    for (size_t i = 0; i < n; ++i) counts[plane[i]]++;
    model_t* m = (model_t*)malloc(sizeof(model_t));
    model_from_counts(m, counts);
    uint8_t* enc = NULL;
    const size_t elen = rans_encode(plane, n, m, &enc);
    put_var(o, (uint32_t)elen);
    uint32_t nused = 0;
    for (int s = 0; s < 256; ++s) nused += m->freq[s] != 0;
    put_var(o, nused);
    for (int s = 0; s < 256; ++s) {
        if (!m->freq[s]) continue;
        buf_push(o, (uint8_t)s);
        put_var(o, m->freq[s]);
    }
    buf_append(o, enc, elen);
    free(enc);
    free(m);
}

/* decode_plane (entropy.hpp:115-155); *out is malloc'd (NULL for an empty plane) */
static int decode_plane(const uint8_t* in, size_t len, size_t* p, uint32_t max_n, uint8_t** out, uint32_t* out_n) {
    uint32_t n, enc_size, nused;
    int e;
    *out = NULL;
    *out_n = 0;
    if ((e = get_var(in, len, p, &n))) return e;
    if (n == 0) return 0;
    if (n > max_n) return E_RANGE;
    if ((e = get_var(in, len, p, &enc_size))) return e;
    if ((e = get_var(in, len, p, &nused))) return e;
    if (nused > 256) return E_RANGE;
    model_t* m = (model_t*)calloc(1, sizeof(model_t));
    for (uint32_t k = 0; k < nused; ++k) {
        if (*p >= len) {
            free(m);
            return E_TRUNC;
        }
        const uint8_t s = in[(*p)++];
        uint32_t f;
        if ((e = get_var(in, len, p, &f))) {
            free(m);
            return e;
        }
        if (f > 0xffffu) {
            free(m);
            return E_RANGE;
        }
        m->freq[s] = (uint16_t)f;
    }
    uint64_t tot = 0;
    for (int s = 0; s < 256; ++s) tot += m->freq[s];
    if (tot != RANS_SCALE) {
        free(m);
        return E_RANGE;
    }
    model_cum(m);
    if (*p + enc_size > len) {
        free(m);
        return E_TRUNC;
    }
    uint8_t* o = (uint8_t*)malloc(n);
    rans_decode(in + *p, enc_size, n, m, o);
    *p += enc_size;
    free(m);
    *out = o;
    *out_n = n;
    return 0;
}

int64_t fxv_encode_plane(const uint8_t* plane, size_t n, uint8_t* out, size_t cap) {
    buf_t o = {0};
    encode_plane(&o, plane, n);
    int64_t r = (int64_t)o.n;
    if (o.oom || o.n > cap) r = -1;
    else memcpy(out, o.b, o.n);
    free(o.b);
    return r;
}

int64_t fxv_decode_plane(const uint8_t* in, size_t len, size_t* pos, uint32_t max_n, uint8_t* out) {
    uint8_t* d;
    uint32_t n;
    const int e = decode_plane(in, len, pos, max_n, &d, &n);
    if (e) return e;
    if (n) memcpy(out, d, n);
    free(d);
    return n;
}

/* ---- LSB-first raw bits (entropy.hpp:159-205) ---- */
typedef struct {
    buf_t o;
    uint64_t acc;
    int nbits;
} bitw_t;

static void bits_put(bitw_t* w, uint32_t v, int bits) {
    if (bits <= 0) return;
    w->acc |= (uint64_t)(v & (bits >= 32 ? 0xffffffffu : ((1u << bits) - 1u))) << w->nbits;
    w->nbits += bits;
    while (w->nbits >= 8) {
        buf_push(&w->o, (uint8_t)(w->acc & 0xffu));
        w->acc >>= 8;
        w->nbits -= 8;
    }
}

static void bits_flush(bitw_t* w) {
    if (w->nbits > 0) {
        buf_push(&w->o, (uint8_t)(w->acc & 0xffu));
        w->acc = 0;
        w->nbits = 0;
    }
}

typedef struct {
    const uint8_t* p;
    size_t n, pos;
    uint64_t acc;
    int nbits;
} bitr_t;

static uint32_t bits_get(bitr_t* r, int bits) {
    if (bits <= 0 || bits > 32) return 0;
    while (r->nbits < bits) {
        r->acc |= (uint64_t)(r->pos < r->n ? r->p[r->pos++] : 0) << r->nbits;
        r->nbits += 8;
    }
    const uint32_t v = (uint32_t)(r->acc & (bits >= 32 ? 0xffffffffu : ((1u << bits) - 1u)));
    r->acc >>= bits;
    r->nbits -= bits;
    return v;
}

/* ---- tile codec helpers (dct_block.hpp:98-128) ---- */
static int32_t causal_pred_s32(const int32_t* a, int bz, int by, int bx) {
    int64_t sum = 0;
    int n = 0;
    if (bx > 0) sum += a[(bz * BPA + by) * BPA + bx - 1], ++n;
    if (by > 0) sum += a[(bz * BPA + by - 1) * BPA + bx], ++n;
    if (bz > 0) sum += a[((bz - 1) * BPA + by) * BPA + bx], ++n;
    return n ? (int32_t)(sum / n) : 0;
}

static int32_t causal_pred_u32(const uint32_t* a, int bz, int by, int bx) {
    int64_t sum = 0;
    int n = 0;
    if (bx > 0) sum += (int64_t)a[(bz * BPA + by) * BPA + bx - 1], ++n;
    if (by > 0) sum += (int64_t)a[(bz * BPA + by - 1) * BPA + bx], ++n;
    if (bz > 0) sum += (int64_t)a[((bz - 1) * BPA + by) * BPA + bx], ++n;
    return n ? (int32_t)(sum / n) : 0;
}

static int raw_ctx(int fsum, int nsum) {
    int band = fsum / 4;
    if (band > BAND_B - 1) band = BAND_B - 1;
    return band * SUM_B + (nsum < SUM_B - 1 ? nsum : SUM_B - 1);
}

static int bit_width(uint32_t a) {
    int w = 0;
    while (a) ++w, a >>= 1;
    return w;
}

static int nsum_of(const uint8_t* sig, scan_e e) {
    const int i = e.idx;
    return ((e.edge & 1) ? sig[i - N * N] : 0) + ((e.edge & 2) ? sig[i - N] : 0) + ((e.edge & 4) ? sig[i - 1] : 0);
}

double fxv_log2_series(double x) {
    int e;
    double m = frexp(x, &e); /* x = m 2^e, m in [1/2, 1) */
    if (m < 0.70710678118654752440) {
        m = m * 2.0;
        e -= 1;
    }
    const double t = (m - 1.0) / (m + 1.0), t2 = t * t;
    double s = 1.0 / 23.0;
    for (int k = 10; k >= 0; --k) {
        const double st = s * t2;
        s = st + 1.0 / (double)(2 * k + 1);
    }
    const double ln_m = (2.0 * t) * s;
    return (double)e + ln_m * 1.4426950408889634;
}

static double lg2(double x, int mode) { return mode ? fxv_log2_series(x) : log2(x); }

/* cluster_contexts cost (dct_block.hpp:176-191) */
static double clust_cost(const uint32_t* h, int mode) {
    double n = 0;
    int nused = 0;
    for (int c = 0; c < NCAT; ++c) {
        n += h[c];
        if (h[c]) ++nused;
    }
    if (n == 0) return 0.0;
    double ent = 0;
    for (int c = 0; c < NCAT; ++c)
        if (h[c]) {
            const double t = (double)h[c] * lg2(n / (double)h[c], mode);
            ent += t;
        }
    return ent + (double)nused * 16.0 + 24.0;
}

/* cluster_contexts (dct_block.hpp:171-257) */
static int cluster_contexts(uint32_t hist[RAW_CTX][NCAT], uint8_t* cluster_of, int mode) {
    uint32_t ch[RAW_CTX][NCAT];
    double ccost[RAW_CTX] = {0};
    int alive[RAW_CTX] = {0};
    int nactive = 0;
    memcpy(ch, hist, sizeof ch);
    for (int r = 0; r < RAW_CTX; ++r) {
        cluster_of[r] = (uint8_t)r;
        double tot = 0;
        for (int c = 0; c < NCAT; ++c) tot += ch[r][c];
        if (tot > 0) {
            alive[r] = 1;
            ccost[r] = clust_cost(ch[r], mode);
            ++nactive;
        }
    }
    if (nactive == 0) {
        memset(cluster_of, 0, RAW_CTX);
        return 1;
    }
    while (nactive > 1) {
        const int force = nactive > MAX_CL;
        double best = 0;
        int bi = -1, bj = -1;
        for (int i = 0; i < RAW_CTX; ++i) {
            if (!alive[i]) continue;
            for (int j = i + 1; j < RAW_CTX; ++j) {
                if (!alive[j]) continue;
                uint32_t mh[NCAT];
                for (int s = 0; s < NCAT; ++s) mh[s] = ch[i][s] + ch[j][s];
                const double d = clust_cost(mh, mode) - ccost[i] - ccost[j];
                if (bi < 0 || d < best) {
                    best = d;
                    bi = i;
                    bj = j;
                }
            }
        }
        if (bi < 0 || (!force && best >= 0)) break;
        for (int s = 0; s < NCAT; ++s) ch[bi][s] += ch[bj][s];
        ccost[bi] = clust_cost(ch[bi], mode);
        alive[bj] = 0;
        for (int r = 0; r < RAW_CTX; ++r)
            if (cluster_of[r] == bj) cluster_of[r] = (uint8_t)bi;
        --nactive;
    }
    int remap[RAW_CTX];
    for (int r = 0; r < RAW_CTX; ++r) remap[r] = -1;
    int K = 0;
    for (int r = 0; r < RAW_CTX; ++r)
        if (alive[cluster_of[r]] && remap[cluster_of[r]] < 0) remap[cluster_of[r]] = K++;
    if (K == 0) K = 1;
    for (int r = 0; r < RAW_CTX; ++r) cluster_of[r] = (uint8_t)(alive[cluster_of[r]] ? remap[cluster_of[r]] : 0);
    return K;
}

/* ---- tile encode (dct_block.hpp:318-484) ---- */
static int64_t encode_tile(const uint8_t* tu8, const float* tf32, const fxv_params* prm, int mode, uint8_t* out,
                           size_t cap) {
    init_tables();
    float stepv[3 * N];
    step_table(prm, stepv);
    int32_t* levall = (int32_t*)malloc(sizeof(int32_t) * NBLK * V);
    float* coefall = (float*)malloc(sizeof(float) * NBLK * V);
    int32_t dclev[NBLK];
    uint32_t nsigs[NBLK];
    uint32_t hist[RAW_CTX][NCAT];
    uint8_t sig[V];
    float c[V];
    memset(hist, 0, sizeof hist);
    const float dc_step = prm->q * 0.0625f;
    for (int b = 0; b < NBLK; ++b) {
        const int bz = b / (BPA * BPA), by = (b / BPA) % BPA, bx = b % BPA;
        int32_t* lev = levall + (size_t)b * V;
        float* coef = coefall + (size_t)b * V;
        /* quant_one_block (dct_block.hpp:131-168) */
        double msum = 0;
        for (int z = 0; z < N; ++z)
            for (int y = 0; y < N; ++y)
                for (int x = 0; x < N; ++x) {
                    const size_t si = ((size_t)(bz * N + z) * SIDE + (by * N + y)) * SIDE + (bx * N + x);
                    const float v = tu8 ? (float)tu8[si] : tf32[si];
                    c[(z * N + y) * N + x] = v;
                    msum += (double)v;
                }
        const float mean = (float)(msum / (double)V);
        const int32_t dl = (int32_t)lroundf(mean / dc_step);
        const float dcv = (float)dl * dc_step;
        for (int i = 0; i < V; ++i) c[i] = c[i] - dcv;
        dct3(c, dct1_fwd);
        for (int z = 0; z < N; ++z)
            for (int y = 0; y < N; ++y)
                for (int x = 0; x < N; ++x) {
                    const int i = (z * N + y) * N + x;
                    const float step = stepv[z + y + x], a0 = fabsf(c[i]);
                    coef[i] = c[i];
                    int32_t level = 0;
                    if (a0 >= prm->dz_frac * step) {
                        const float t = a0 / step + (1.0f - prm->dz_frac);
                        level = (c[i] < 0 ? -1 : 1) * (int32_t)floorf(t);
                    }
                    lev[i] = level < -32768 ? -32768 : (level > 32767 ? 32767 : level);
                }
        uint32_t ns = 0;
        for (int pos = V - 1; pos >= 0; --pos)
            if (lev[g_scan[pos].idx] != 0) {
                ns = (uint32_t)(pos + 1);
                break;
            }
        dclev[b] = dl;
        nsigs[b] = ns;
        memset(sig, 0, V);
        for (uint32_t pos = 0; pos < ns; ++pos) {
            const scan_e e = g_scan[pos];
            const int nsum = nsum_of(sig, e);
            const uint32_t a = (uint32_t)(lev[e.idx] < 0 ? -lev[e.idx] : lev[e.idx]);
            const int cat = a ? bit_width(a) : 0;
            hist[raw_ctx(e.fsum, nsum)][cat]++;
            sig[e.idx] = (uint8_t)(a < MAG_CAP ? a : MAG_CAP);
        }
    }
    uint8_t cmap[RAW_CTX];
    const int K = cluster_contexts(hist, cmap, mode);

    if (prm->rdoq) { /* dct_block.hpp:357-413 */
        float bc[MAX_CL][NCAT];
        double chist[MAX_CL][NCAT];
        memset(bc, 0, sizeof bc);
        memset(chist, 0, sizeof chist);
        for (int r = 0; r < RAW_CTX; ++r)
            for (int cat = 0; cat < NCAT; ++cat) chist[cmap[r]][cat] += hist[r][cat];
        for (int cl = 0; cl < K; ++cl) {
            double tot = 0;
            for (int cat = 0; cat < NCAT; ++cat) tot += chist[cl][cat];
            for (int cat = 0; cat < NCAT; ++cat)
                bc[cl][cat] = (float)(-lg2((chist[cl][cat] + 0.5) / (tot + 0.5 * NCAT), mode));
        }
        for (int b = 0; b < NBLK; ++b) {
            int32_t* lev = levall + (size_t)b * V;
            const float* coef = coefall + (size_t)b * V;
            memset(sig, 0, V);
            for (uint32_t pos = 0; pos < nsigs[b]; ++pos) {
                const scan_e e = g_scan[pos];
                const int i = e.idx;
                const uint32_t m0 = (uint32_t)(lev[i] < 0 ? -lev[i] : lev[i]);
                if (m0 == 0) {
                    sig[i] = 0;
                    continue;
                }
                const int cl = cmap[raw_ctx(e.fsum, nsum_of(sig, e))];
                const float s = stepv[e.fsum], lam = prm->rdoq_lambda * s * s, ac = fabsf(coef[i]);
#define RD(m, outv)                                                                                   \
    do {                                                                                              \
        const uint32_t m_ = (m);                                                                      \
        const float dq_ = m_ ? s * ((float)m_ - 1.0f + prm->dz_frac + 0.40f) : 0.0f;                  \
        const int cat_ = m_ ? bit_width(m_) : 0;                                                      \
        const float df_ = ac - dq_;                                                                   \
        const float d2_ = df_ * df_;                                                                  \
        const float r_ = lam * (bc[cl][cat_] + (float)(m_ ? cat_ : 0));                               \
        (outv) = d2_ + r_;                                                                            \
    } while (0)
                uint32_t bm = m0;
                float best, c0, c1;
                RD(m0, best);
                RD(0, c0);
                if (c0 < best) {
                    best = c0;
                    bm = 0;
                }
                if (m0 >= 2) {
                    RD(m0 - 1, c1);
                    if (c1 < best) {
                        best = c1;
                        bm = m0 - 1;
                    }
                }
#undef RD
                lev[i] = lev[i] < 0 ? -(int32_t)bm : (int32_t)bm;
                sig[i] = (uint8_t)(bm < MAG_CAP ? bm : MAG_CAP);
            }
            uint32_t n2 = 0;
            for (int pos = (int)nsigs[b] - 1; pos >= 0; --pos)
                if (lev[g_scan[pos].idx] != 0) {
                    n2 = (uint32_t)(pos + 1);
                    break;
                }
            nsigs[b] = n2;
        }
    }

    /* phase B (dct_block.hpp:415-439) */
    buf_t cats[MAX_CL];
    memset(cats, 0, sizeof cats);
    bitw_t bits;
    memset(&bits, 0, sizeof bits);
    for (int b = 0; b < NBLK; ++b) {
        const int32_t* lev = levall + (size_t)b * V;
        memset(sig, 0, V);
        for (uint32_t pos = 0; pos < nsigs[b]; ++pos) {
            const scan_e e = g_scan[pos];
            const int cl = cmap[raw_ctx(e.fsum, nsum_of(sig, e))];
            const int32_t level = lev[e.idx];
            const uint32_t a = (uint32_t)(level < 0 ? -level : level);
            const int cat = a ? bit_width(a) : 0;
            buf_push(&cats[cl], (uint8_t)cat);
            sig[e.idx] = (uint8_t)(a < MAG_CAP ? a : MAG_CAP);
            if (cat > 0) {
                bits_put(&bits, a - (1u << (cat - 1)), cat - 1);
                bits_put(&bits, level < 0 ? 1u : 0u, 1);
            }
        }
    }
    buf_t o = {0};
    for (int b = 0; b < NBLK; ++b) {
        const int bz = b / (BPA * BPA), by = (b / BPA) % BPA, bx = b % BPA;
        const int32_t pred = prm->dc_predict ? causal_pred_s32(dclev, bz, by, bx) : 0;
        const int32_t res = dclev[b] - pred;
        put_var(&o, ((uint32_t)res << 1) ^ (uint32_t)(res >> 31));
    }
    for (int b = 0; b < NBLK; ++b) {
        const int bz = b / (BPA * BPA), by = (b / BPA) % BPA, bx = b % BPA;
        const int32_t pred = prm->dc_predict ? causal_pred_u32(nsigs, bz, by, bx) : 0;
        const int32_t res = (int32_t)nsigs[b] - pred;
        put_var(&o, ((uint32_t)res << 1) ^ (uint32_t)(res >> 31));
    }
    buf_push(&o, (uint8_t)K);
    buf_append(&o, cmap, RAW_CTX);
    for (int cl = 0; cl < K; ++cl) encode_plane(&o, cats[cl].b, cats[cl].n);
    bits_flush(&bits);
    put_var(&o, (uint32_t)bits.o.n);
    buf_append(&o, bits.o.b, bits.o.n);

    int64_t r = (int64_t)o.n;
    int oom = o.oom || bits.o.oom;
    for (int cl = 0; cl < MAX_CL; ++cl) oom |= cats[cl].oom, free(cats[cl].b);
    if (oom) r = E_NOMEM;
    else if (o.n > cap) r = -1;
    else memcpy(out, o.b, o.n);
    free(o.b);
    free(bits.o.b);
    free(levall);
    free(coefall);
    return r;
}

int64_t fxv_encode_tile_u8(const uint8_t* tile, const fxv_params* p, int log2_mode, uint8_t* out, size_t cap) {
    return encode_tile(tile, NULL, p, log2_mode, out, cap);
}

int64_t fxv_encode_tile_f32(const float* tile, const fxv_params* p, int log2_mode, uint8_t* out, size_t cap) {
    return encode_tile(NULL, tile, p, log2_mode, out, cap);
}

/* quant-gated deblock (dct_block.hpp:267-309), the reference's sequential order */
static void smooth(float p2, float p1, float* p0, float* q0, float q1, float q2, float beta, float tc) {
    const float dp = fabsf(p2 - 2.0f * p1 + *p0), dq = fabsf(q2 - 2.0f * q1 + *q0);
    if (dp + dq >= beta) return;
    float delta = (9.0f * (*q0 - *p0) - 3.0f * (q1 - p1)) * (1.0f / 16.0f);
    if (fabsf(delta) >= 10.0f * tc) return;
    if (delta < -tc) delta = -tc;
    else if (tc < delta) delta = tc;
    *p0 += delta;
    *q0 -= delta;
}

static void deblock_tile(float* t, const fxv_params* p) {
    const float beta = p->deblock_beta * p->q, tc = p->deblock_tc * p->q;
    if (tc <= 0.0f) return;
#define AT(z, y, x) t[((size_t)(z)*SIDE + (y)) * SIDE + (x)]
    for (int b = N; b < SIDE; b += N)
        for (int i = 0; i < SIDE; ++i)
            for (int j = 0; j < SIDE; ++j) {
                smooth(AT(b - 3, i, j), AT(b - 2, i, j), &AT(b - 1, i, j), &AT(b, i, j), AT(b + 1, i, j),
                       AT(b + 2, i, j), beta, tc);
                smooth(AT(i, b - 3, j), AT(i, b - 2, j), &AT(i, b - 1, j), &AT(i, b, j), AT(i, b + 1, j),
                       AT(i, b + 2, j), beta, tc);
                smooth(AT(i, j, b - 3), AT(i, j, b - 2), &AT(i, j, b - 1), &AT(i, j, b), AT(i, j, b + 1),
                       AT(i, j, b + 2), beta, tc);
            }
#undef AT
}

/* ---- tile decode (dct_block.hpp:492-588) ---- */
int fxv_decode_tile(const uint8_t* payload, size_t len, const fxv_params* prm, float* recon_out, uint8_t* out_u8) {
    init_tables();
    size_t p = 0;
    int32_t dclev[NBLK];
    uint32_t nsigs[NBLK];
    int e;
    uint32_t zz;
    for (int b = 0; b < NBLK; ++b) {
        if ((e = get_var(payload, len, &p, &zz))) return e;
        const int32_t res = (int32_t)(zz >> 1) ^ -(int32_t)(zz & 1u);
        const int bz = b / (BPA * BPA), by = (b / BPA) % BPA, bx = b % BPA;
        const int32_t pred = prm->dc_predict ? causal_pred_s32(dclev, bz, by, bx) : 0;
        dclev[b] = (int32_t)((uint32_t)res + (uint32_t)pred);
    }
    for (int b = 0; b < NBLK; ++b) {
        if ((e = get_var(payload, len, &p, &zz))) return e;
        const int32_t res = (int32_t)(zz >> 1) ^ -(int32_t)(zz & 1u);
        const int bz = b / (BPA * BPA), by = (b / BPA) % BPA, bx = b % BPA;
        const int32_t pred = prm->dc_predict ? causal_pred_u32(nsigs, bz, by, bx) : 0;
        const int64_t ns = (int64_t)res + pred;
        if (ns < 0 || ns > V) return E_RANGE;
        nsigs[b] = (uint32_t)ns;
    }
    if (p >= len) return E_TRUNC;
    const int K = payload[p++];
    if (K <= 0 || K > MAX_CL) return E_RANGE;
    if (p + RAW_CTX > len) return E_TRUNC;
    uint8_t cmap[RAW_CTX];
    for (int r = 0; r < RAW_CTX; ++r) {
        const uint8_t v = payload[p++];
        if (v >= K) return E_RANGE;
        cmap[r] = v;
    }
    uint8_t* cats[MAX_CL] = {0};
    uint32_t ncat[MAX_CL] = {0}, cur[MAX_CL] = {0};
    int rc = 0;
    float* recon = NULL;
    for (int cl = 0; cl < K && !rc; ++cl) {
        rc = decode_plane(payload, len, &p, (uint32_t)(NBLK * V), &cats[cl], &ncat[cl]);
        for (uint32_t i = 0; !rc && i < ncat[cl]; ++i)
            if (cats[cl][i] >= NCAT) rc = E_RANGE;
    }
    uint32_t nb = 0;
    if (!rc) rc = get_var(payload, len, &p, &nb);
    if (!rc && p + nb > len) rc = E_TRUNC;
    if (!rc) {
        bitr_t bits = {payload + p, nb, 0, 0, 0};
        p += nb;
        float stepv[3 * N];
        step_table(prm, stepv);
        recon = (float*)malloc(sizeof(float) * SIDE * SIDE * SIDE);
        float c[V];
        uint8_t sig[V];
        for (int b = 0; b < NBLK && !rc; ++b) {
            const int bz = b / (BPA * BPA), by = (b / BPA) % BPA, bx = b % BPA;
            memset(c, 0, sizeof c);
            memset(sig, 0, sizeof sig);
            const float dc = (float)dclev[b] * (prm->q * 0.0625f);
            for (uint32_t pos = 0; pos < nsigs[b]; ++pos) {
                const scan_e se = g_scan[pos];
                const int cl = cmap[raw_ctx(se.fsum, nsum_of(sig, se))];
                if (cur[cl] >= ncat[cl]) {
                    rc = E_UNDERRUN;
                    break;
                }
                const int cat = cats[cl][cur[cl]++];
                if (cat > 0) {
                    const uint32_t a = (1u << (cat - 1)) + bits_get(&bits, cat - 1);
                    const int neg = bits_get(&bits, 1) != 0;
                    const float mag = stepv[se.fsum] * ((float)a - 1.0f + prm->dz_frac + 0.40f);
                    c[se.idx] = neg ? -mag : mag;
                    sig[se.idx] = (uint8_t)(a < MAG_CAP ? a : MAG_CAP);
                }
            }
            if (rc) break;
            dct3(c, dct1_inv);
            for (int z = 0; z < N; ++z)
                for (int y = 0; y < N; ++y)
                    for (int x = 0; x < N; ++x)
                        recon[((size_t)(bz * N + z) * SIDE + (by * N + y)) * SIDE + (bx * N + x)] =
                            c[(z * N + y) * N + x] + dc;
        }
    }
    for (int cl = 0; cl < MAX_CL; ++cl) free(cats[cl]);
    if (rc) {
        free(recon);
        return rc;
    }
    if (prm->deblock) deblock_tile(recon, prm);
    const size_t nv = (size_t)SIDE * SIDE * SIDE;
    if (recon_out) memcpy(recon_out, recon, nv * sizeof(float));
    if (out_u8)
        for (size_t i = 0; i < nv; ++i) {
            double r = nearbyint((double)recon[i]);
            r = r < 0.0 ? 0.0 : (r > 255.0 ? 255.0 : r);
            out_u8[i] = (uint8_t)r;
        }
    free(recon);
    return 0;
}

/* ---- container helpers (archive.hpp:47-74) ---- */
uint32_t fxv_crc32c(const uint8_t* p, size_t n) {
    static uint32_t table[256];
    static int ready;
    if (!ready) {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ 0x82f63b78u : c >> 1;
            table[i] = c;
        }
        ready = 1;
    }
    uint32_t crc = ~0u;
    for (size_t i = 0; i < n; ++i) crc = table[(crc ^ p[i]) & 0xffu] ^ (crc >> 8);
    return ~crc;
}

static uint64_t part1by2(uint64_t x) {
    x &= 0x1fffffull;
    x = (x | (x << 32)) & 0x1f00000000ffffull;
    x = (x | (x << 16)) & 0x1f0000ff0000ffull;
    x = (x | (x << 8)) & 0x100f00f00f00f00full;
    x = (x | (x << 4)) & 0x10c30c30c30c30c3ull;
    x = (x | (x << 2)) & 0x1249249249249249ull;
    return x;
}

uint64_t fxv_morton3(uint64_t z, uint64_t y, uint64_t x) {
    return (part1by2(z) << 2) | (part1by2(y) << 1) | part1by2(x);
}
