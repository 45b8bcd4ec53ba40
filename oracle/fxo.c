/* fxo.c — CPU oracle (test infrastructure only). See fxo.h for what each part restates.
 * Build: gcc -O2 -fopenmp -ffp-contract=off (no fast-math, no FMA contraction: the tiling
 * weights and the blend normalisation are compared bit-exactly). */
#include "fxo.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ---- tiling: src/ml/tiling.hpp:16-42, src/ml/infer.hpp:499-509 ------------------------------ */
int64_t fxo_tile_starts(int64_t dim, int patch, double overlap, int64_t* out, int64_t cap) {
    int64_t n = 0;
    if (dim <= patch) {
        if (cap > 0) out[0] = 0;
        return 1;
    }
    int64_t step = (int64_t)(patch * (1.0 - overlap));
    if (step < 1) step = 1;
    int64_t last = -1;
    for (int64_t s = 0;; s += step) {
        const int64_t c = s < dim - patch ? s : dim - patch;
        if (n == 0 || last != c) {
            if (n < cap) out[n] = c;
            ++n;
            last = c;
        }
        if (c == dim - patch) break;
    }
    return n;
}

void fxo_gaussian1d(int n, float* out) {
    const double c = (n - 1) / 2.0, sigma = n / 8.0;
    double mx = 0.0;
    for (int i = 0; i < n; ++i) {
        const double dd = (i - c) / sigma;
        out[i] = (float)exp(-0.5 * dd * dd);
        if ((double)out[i] > mx) mx = (double)out[i];
    }
    for (int i = 0; i < n; ++i) {
        const float v = (float)(out[i] / mx);
        out[i] = v > 0.1f ? v : 0.1f;
    }
}

void fxo_weight_profile(const float* g, int patch, const int64_t* starts, int64_t nstarts, int64_t c0, int64_t cn,
                        int64_t dim, float* out) {
    for (int64_t i = 0; i < cn; ++i) out[i] = 0.0f;
    for (int64_t k = 0; k < nstarts; ++k) {
        const int64_t s0 = starts[k];
        for (int i = 0; i < patch && s0 + i < dim; ++i) {
            const int64_t gc = s0 + i;
            if (gc >= c0 && gc < c0 + cn) out[gc - c0] += g[i];
        }
    }
}

/* ---- patch fill + z-score: src/ml/inference.cpp:309-321, src/ml/infer.hpp:350-385 ----------- */
static int64_t clampi(int64_t v, int64_t lo, int64_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

void fxo_fill_tile_u8(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, int64_t z0, int64_t y0, int64_t x0,
                      int tz, int ty, int tx, float* out) {
#pragma omp parallel for
    for (int z = 0; z < tz; ++z)
        for (int y = 0; y < ty; ++y)
            for (int x = 0; x < tx; ++x) {
                const int64_t zz = clampi(z0 + z, 0, dz - 1), yy = clampi(y0 + y, 0, dy - 1),
                              xx = clampi(x0 + x, 0, dx - 1);
                out[((int64_t)z * ty + y) * tx + x] = (float)vol[(zz * dy + yy) * dx + xx];
            }
}

void fxo_fill_patch_u8(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, int64_t z0, int64_t y0, int64_t x0,
                       int P, float* out) {
    fxo_fill_tile_u8(vol, dz, dy, dx, z0, y0, x0, P, P, P, out);
}

void fxo_norm_tile_zscore(float* x, int tz, int ty, int tx) {
    const int64_t PN = (int64_t)tz * ty * tx;
    const int64_t pl = (int64_t)ty * tx;
    double* psum = (double*)calloc((size_t)tz, sizeof(double));
    double* psq = (double*)calloc((size_t)tz, sizeof(double));
#pragma omp parallel for
    for (int z = 0; z < tz; ++z) {
        double ls = 0.0, lq = 0.0;
        const float* row = x + (int64_t)z * pl;
        for (int64_t i = 0; i < pl; ++i) {
            const double v = row[i];
            ls += v;
            lq += v * v;
        }
        psum[z] = ls;
        psq[z] = lq;
    }
    double sum = 0.0, sq = 0.0;
    for (int z = 0; z < tz; ++z) {
        sum += psum[z];
        sq += psq[z];
    }
    free(psum);
    free(psq);
    const double n = (double)PN;
    const double mean = sum / n;
    double var = sq / n - mean * mean;
    if (var < 1e-12) var = 1e-12;
    const double sd = sqrt(var);
#pragma omp parallel for
    for (int64_t i = 0; i < PN; ++i) x[i] = (float)((x[i] - mean) / sd);
}

void fxo_norm_patch_zscore(float* x, int P) { fxo_norm_tile_zscore(x, P, P, P); }

/* ---- conv3d 3x3x3, zero padding 1, stride 1|2 per axis (torch.nn.Conv3d semantics) -------- */
void fxo_conv3d_s(const float* x, int B, int Cin, int D, int H, int W, const float* w, const float* bias, int Cout,
                  int sz, int sy, int sx, float* y) {
    const int Do = (D + 2 - 3) / sz + 1, Ho = (H + 2 - 3) / sy + 1, Wo = (W + 2 - 3) / sx + 1;
    const int64_t vin = (int64_t)D * H * W, vout = (int64_t)Do * Ho * Wo;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int b = 0; b < B; ++b)
        for (int co = 0; co < Cout; ++co) {
            float* yo = y + ((int64_t)b * Cout + co) * vout;
            const float bv = bias ? bias[co] : 0.0f;
            for (int64_t i = 0; i < vout; ++i) yo[i] = 0.0f;
            for (int ci = 0; ci < Cin; ++ci) {
                const float* xi = x + ((int64_t)b * Cin + ci) * vin;
                for (int kz = 0; kz < 3; ++kz)
                    for (int ky = 0; ky < 3; ++ky)
                        for (int kx = 0; kx < 3; ++kx) {
                            const float wv = w[(((int64_t)co * Cin + ci) * 3 + kz) * 9 + ky * 3 + kx];
                            for (int zo = 0; zo < Do; ++zo) {
                                const int zi = zo * sz - 1 + kz;
                                if (zi < 0 || zi >= D) continue;
                                for (int yo_ = 0; yo_ < Ho; ++yo_) {
                                    const int yi = yo_ * sy - 1 + ky;
                                    if (yi < 0 || yi >= H) continue;
                                    const float* xr = xi + ((int64_t)zi * H + yi) * W;
                                    float* yr = yo + ((int64_t)zo * Ho + yo_) * Wo;
                                    if (sx == 1) {
                                        const int lo = kx == 0 ? 1 : 0, hi = kx == 2 ? Wo - 1 : Wo;
                                        const float* xs = xr + kx - 1;
                                        for (int xo = lo; xo < hi; ++xo) yr[xo] += wv * xs[xo];
                                    } else {
                                        for (int xo = 0; xo < Wo; ++xo) {
                                            const int xx = xo * sx - 1 + kx;
                                            if (xx >= 0 && xx < W) yr[xo] += wv * xr[xx];
                                        }
                                    }
                                }
                            }
                        }
            }
            if (bv != 0.0f)
                for (int64_t i = 0; i < vout; ++i) yo[i] += bv;
        }
}

void fxo_conv3d(const float* x, int B, int Cin, int D, int H, int W, const float* w, const float* bias, int Cout,
                int stride, float* y) {
    fxo_conv3d_s(x, B, Cin, D, H, W, w, bias, Cout, stride, stride, stride, y);
}

/* ---- InstanceNorm3d(affine, eps) + LeakyReLU: resenc_unet.hpp:35-52 ------------------------- */
void fxo_instance_norm_act(float* x, int B, int C, int64_t S, const float* gamma, const float* beta, float eps,
                           int act, float slope) {
#pragma omp parallel for collapse(2)
    for (int b = 0; b < B; ++b)
        for (int c = 0; c < C; ++c) {
            float* p = x + ((int64_t)b * C + c) * S;
            double m = 0.0;
            for (int64_t i = 0; i < S; ++i) m += p[i];
            m /= (double)S;
            double v = 0.0;
            for (int64_t i = 0; i < S; ++i) {
                const double d = p[i] - m;
                v += d * d;
            }
            v /= (double)S; /* biased */
            const float inv = (float)(1.0 / sqrt(v + (double)eps));
            const float g = gamma ? gamma[c] : 1.0f, bb = beta ? beta[c] : 0.0f;
            const float mf = (float)m;
            for (int64_t i = 0; i < S; ++i) {
                float t = (p[i] - mf) * inv * g + bb;
                if (act && t < 0.0f) t *= slope;
                p[i] = t;
            }
        }
}

/* ---- ConvTranspose3d(kernel = stride = (kz, ky, kx), each 1 or 2) with bias: resenc_unet.hpp:211
 * (kernel 2, stride 2 there; nnU-Net sets both to the stage's per-axis pooling kernel) --------- */
void fxo_conv_transpose_s(const float* x, int B, int Cin, int D, int H, int W, const float* w, const float* bias,
                          int Cout, int kz, int ky, int kx, float* y) {
    const int64_t vin = (int64_t)D * H * W;
    const int Do = kz * D, Ho = ky * H, Wo = kx * W, nk = kz * ky * kx;
    const int64_t vout = (int64_t)Do * Ho * Wo;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int b = 0; b < B; ++b)
        for (int co = 0; co < Cout; ++co) {
            float* yo = y + ((int64_t)b * Cout + co) * vout;
            for (int64_t i = 0; i < vout; ++i) yo[i] = bias ? bias[co] : 0.0f;
            for (int ci = 0; ci < Cin; ++ci) {
                const float* xi = x + ((int64_t)b * Cin + ci) * vin;
                const float* wk = w + ((int64_t)ci * Cout + co) * nk;
                for (int z = 0; z < D; ++z)
                    for (int yy = 0; yy < H; ++yy) {
                        const float* xr = xi + ((int64_t)z * H + yy) * W;
                        for (int az = 0; az < kz; ++az)
                            for (int ay = 0; ay < ky; ++ay) {
                                float* yr = yo + ((int64_t)(kz * z + az) * Ho + (ky * yy + ay)) * Wo;
                                for (int ax = 0; ax < kx; ++ax) {
                                    const float wv = wk[(az * ky + ay) * kx + ax];
                                    for (int xx = 0; xx < W; ++xx) yr[kx * xx + ax] += wv * xr[xx];
                                }
                            }
                    }
            }
        }
}

void fxo_conv_transpose2(const float* x, int B, int Cin, int D, int H, int W, const float* w, const float* bias,
                         int Cout, float* y) {
    fxo_conv_transpose_s(x, B, Cin, D, H, W, w, bias, Cout, 2, 2, 2, y);
}

/* ---- 1x1x1 head + softmax channel select / sigmoid + nan_to_num: infer.hpp:760-767 -------- */
void fxo_head(const float* x, int B, int C, int64_t S, const float* w, const float* b, int ncls, int channel,
              int sigmoid, float* prob) {
#pragma omp parallel for collapse(2)
    for (int bb = 0; bb < B; ++bb)
        for (int64_t i = 0; i < S; ++i) {
            float l[8];
            for (int k = 0; k < ncls; ++k) {
                float acc = b[k];
                for (int c = 0; c < C; ++c) acc += w[k * C + c] * x[((int64_t)bb * C + c) * S + i];
                l[k] = acc;
            }
            float p;
            if (sigmoid) {
                p = 1.0f / (1.0f + expf(-l[0]));
            } else {
                float m = l[0];
                for (int k = 1; k < ncls; ++k) m = l[k] > m ? l[k] : m;
                float den = 0.0f, num = 0.0f;
                for (int k = 0; k < ncls; ++k) {
                    const float e = expf(l[k] - m);
                    den += e;
                    if (k == channel) num = e;
                }
                p = num / den;
            }
            if (isnan(p)) p = 0.0f;
            else if (isinf(p)) p = p > 0 ? 1.0f : 0.0f;
            prob[(int64_t)bb * S + i] = p;
        }
}

/* ---- .fxweights (src/ml/weights.hpp:1-10, 63-123) -------------------------------------- */
typedef struct {
    char* name;
    int ndim;
    int64_t shape[8];
    float* data;
    int64_t numel;
} fxo_tensor;

struct fxo_net {
    fxo_tensor* t;
    int nt;
    int S, nconv, ncls;
    int F[16];
    int st[16][3]; /* per stage: stride (z, y, x) of its first conv = kernel of the transposed conv undoing it */
};

static const fxo_tensor* find_t(const fxo_net* n, const char* name) {
    for (int i = 0; i < n->nt; ++i)
        if (strcmp(n->t[i].name, name) == 0) return &n->t[i];
    return NULL;
}

void fxo_net_free(fxo_net* n) {
    if (!n) return;
    for (int i = 0; i < n->nt; ++i) {
        free(n->t[i].name);
        free(n->t[i].data);
    }
    free(n->t);
    free(n);
}

static float bf16_to_f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

fxo_net* fxo_net_load(const char* path) {
    FILE* f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    const long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    uint8_t* buf = (uint8_t*)malloc((size_t)sz);
    if (!buf || fread(buf, 1, (size_t)sz, f) != (size_t)sz) {
        fclose(f);
        free(buf);
        return NULL;
    }
    fclose(f);
    fxo_net* n = (fxo_net*)calloc(1, sizeof(fxo_net));
    uint32_t ver = 0, cnt = 0;
    if (sz < 16 || memcmp(buf, "FXWT", 4) != 0) goto bad;
    memcpy(&ver, buf + 4, 4);
    memcpy(&cnt, buf + 8, 4);
    if (ver != 1) goto bad;
    n->t = (fxo_tensor*)calloc(cnt, sizeof(fxo_tensor));
    {
        size_t cur = 16;
        for (uint32_t i = 0; i < cnt; ++i) {
            uint16_t nl;
            if (cur + 2 > (size_t)sz) goto bad;
            memcpy(&nl, buf + cur, 2);
            cur += 2;
            if (cur + nl + 18 > (size_t)sz) goto bad;
            fxo_tensor* t = &n->t[n->nt++];
            t->name = (char*)malloc(nl + 1u);
            memcpy(t->name, buf + cur, nl);
            t->name[nl] = 0;
            cur += nl;
            const uint8_t dt = buf[cur], nd = buf[cur + 1];
            cur += 2;
            uint64_t nbytes, off;
            memcpy(&nbytes, buf + cur, 8);
            memcpy(&off, buf + cur + 8, 8);
            cur += 16;
            if (nd > 8 || cur + 8u * nd > (size_t)sz) goto bad;
            t->ndim = nd;
            t->numel = 1;
            for (int d = 0; d < nd; ++d) {
                memcpy(&t->shape[d], buf + cur, 8);
                cur += 8;
                t->numel *= t->shape[d];
            }
            if (off > (uint64_t)sz || nbytes > (uint64_t)sz - off) goto bad;
            t->data = (float*)malloc(sizeof(float) * (size_t)(t->numel ? t->numel : 1));
            if (dt == 0 && nbytes == 4u * (uint64_t)t->numel) {
                memcpy(t->data, buf + off, nbytes);
            } else if (dt == 2 && nbytes == 2u * (uint64_t)t->numel) {
                for (int64_t k = 0; k < t->numel; ++k) {
                    uint16_t h;
                    memcpy(&h, buf + off + 2 * k, 2);
                    t->data[k] = bf16_to_f(h);
                }
            } else {
                goto bad;
            }
        }
    }
    free(buf);
    buf = NULL;
    {
        char nm[256];
        n->S = 0;
        for (;;) {
            snprintf(nm, sizeof nm, "encoder.stages.%d.convs.0.conv.weight", n->S);
            const fxo_tensor* t = find_t(n, nm);
            if (!t) break;
            n->F[n->S++] = (int)t->shape[0];
            if (n->S >= 16) break;
        }
        n->nconv = 0;
        for (;;) {
            snprintf(nm, sizeof nm, "encoder.stages.0.convs.%d.conv.weight", n->nconv);
            if (!find_t(n, nm)) break;
            ++n->nconv;
        }
        snprintf(nm, sizeof nm, "decoder.seg_layers.%d.weight", n->S - 2);
        const fxo_tensor* h = find_t(n, nm);
        if (n->S < 2 || n->nconv < 1 || !h) goto bad;
        n->ncls = (int)h->shape[0];
        n->st[0][0] = n->st[0][1] = n->st[0][2] = 1;
        for (int s = 1; s < n->S; ++s) {
            snprintf(nm, sizeof nm, "decoder.transpconvs.%d.weight", n->S - 1 - s);
            const fxo_tensor* tp = find_t(n, nm);
            if (!tp || tp->ndim != 5) goto bad;
            for (int a = 0; a < 3; ++a) {
                if (tp->shape[2 + a] != 1 && tp->shape[2 + a] != 2) goto bad;
                n->st[s][a] = (int)tp->shape[2 + a];
            }
        }
    }
    return n;
bad:
    free(buf);
    fxo_net_free(n);
    return NULL;
}

int fxo_net_stages(const fxo_net* n) { return n ? n->S : 0; }

static const float* W_(const fxo_net* n, const char* fmt, int a, int b) {
    char nm[256];
    snprintf(nm, sizeof nm, fmt, a, b);
    const fxo_tensor* t = find_t(n, nm);
    return t ? t->data : NULL;
}

/* ConvNormAct: conv(k3, pad 1, stride, bias) -> InstanceNorm3d(affine, eps 1e-5) -> LeakyReLU(0.01);
 * g = the input extents (z, y, x), replaced by the output's */
static float* conv_norm_act(const fxo_net* n, const char* pre, int idx, int i, const float* x, int B, int Cin,
                            int g[3], const int stride[3], int Cout) {
    char fw[256], fb[256], fg[256], fbt[256];
    snprintf(fw, sizeof fw, "%s.%%d.convs.%%d.conv.weight", pre);
    snprintf(fb, sizeof fb, "%s.%%d.convs.%%d.conv.bias", pre);
    snprintf(fg, sizeof fg, "%s.%%d.convs.%%d.norm.weight", pre);
    snprintf(fbt, sizeof fbt, "%s.%%d.convs.%%d.norm.bias", pre);
    const int o[3] = {g[0] / stride[0], g[1] / stride[1], g[2] / stride[2]};
    const int64_t S = (int64_t)o[0] * o[1] * o[2];
    float* y = (float*)malloc(sizeof(float) * (size_t)(B * (int64_t)Cout * S));
    fxo_conv3d_s(x, B, Cin, g[0], g[1], g[2], W_(n, fw, idx, i), W_(n, fb, idx, i), Cout, stride[0], stride[1], stride[2],
                 y);
    fxo_instance_norm_act(y, B, Cout, S, W_(n, fg, idx, i), W_(n, fbt, idx, i), 1e-5f, 1, 0.01f);
    for (int a = 0; a < 3; ++a) g[a] = o[a];
    return y;
}

int fxo_net_tile_ok(const fxo_net* n, int tz, int ty, int tx) {
    int g[3] = {tz, ty, tx};
    if (tz < 1 || ty < 1 || tx < 1) return 0;
    for (int s = 1; s < n->S; ++s)
        for (int a = 0; a < 3; ++a) {
            if (g[a] % n->st[s][a]) return 0;
            g[a] /= n->st[s][a];
        }
    return 1;
}

int fxo_net_forward_tiled(const fxo_net* n, const float* x, int B, int tz, int ty, int tx, int channel, int sigmoid,
                          float* prob) {
    if (!fxo_net_tile_ok(n, tz, ty, tx)) return 1;
    const int S = n->S;
    static const int one[3] = {1, 1, 1};
    float* skips[16] = {0};
    const int64_t v0 = (int64_t)tz * ty * tx;
    float* cur = (float*)malloc(sizeof(float) * (size_t)(B * v0));
    memcpy(cur, x, sizeof(float) * (size_t)(B * v0));
    int C = 1, g[3] = {tz, ty, tx};
    /* encoder: ConvStack(prev, F[s], 3, stride[s], nconv) per stage */
    for (int s = 0; s < S; ++s)
        for (int i = 0; i < n->nconv; ++i) {
            float* y = conv_norm_act(n, "encoder.stages", s, i, cur, B, C, g, i == 0 ? n->st[s] : one, n->F[s]);
            free(cur);
            cur = y;
            C = n->F[s];
            if (i == n->nconv - 1) {
                const int64_t sz = (int64_t)B * C * g[0] * g[1] * g[2];
                skips[s] = (float*)malloc(sizeof(float) * (size_t)sz);
                memcpy(skips[s], cur, sizeof(float) * (size_t)sz);
            }
        }
    /* decoder: transpconv -> cat(up, skip) -> ConvStack(2 F, F, 3, 1, nconv) (resenc_unet.hpp:227-237) */
    for (int t = 0; t < S - 1; ++t) {
        const int lvl = S - 2 - t, F = n->F[lvl];
        const int* k = n->st[lvl + 1];
        const int gn[3] = {g[0] * k[0], g[1] * k[1], g[2] * k[2]};
        const int64_t S3 = (int64_t)gn[0] * gn[1] * gn[2];
        float* up = (float*)malloc(sizeof(float) * (size_t)(B * (int64_t)F * S3));
        fxo_conv_transpose_s(cur, B, C, g[0], g[1], g[2], W_(n, "decoder.transpconvs.%d.weight", t, 0),
                             W_(n, "decoder.transpconvs.%d.bias", t, 0), F, k[0], k[1], k[2], up);
        float* cat = (float*)malloc(sizeof(float) * (size_t)(B * (int64_t)2 * F * S3));
        for (int b = 0; b < B; ++b) {
            memcpy(cat + (int64_t)b * 2 * F * S3, up + (int64_t)b * F * S3, sizeof(float) * (size_t)(F * S3));
            memcpy(cat + ((int64_t)b * 2 + 1) * F * S3, skips[lvl] + (int64_t)b * F * S3,
                   sizeof(float) * (size_t)(F * S3));
        }
        free(up);
        free(cur);
        cur = cat;
        C = 2 * F;
        for (int a = 0; a < 3; ++a) g[a] = gn[a];
        for (int i = 0; i < n->nconv; ++i) {
            float* y = conv_norm_act(n, "decoder.stages", t, i, cur, B, C, g, one, F);
            free(cur);
            cur = y;
            C = F;
        }
    }
    const int64_t S3 = (int64_t)g[0] * g[1] * g[2];
    fxo_head(cur, B, C, S3, W_(n, "decoder.seg_layers.%d.weight", S - 2, 0), W_(n, "decoder.seg_layers.%d.bias", S - 2, 0),
             n->ncls, channel, sigmoid, prob);
    free(cur);
    for (int s = 0; s < S; ++s) free(skips[s]);
    return 0;
}

int fxo_net_forward(const fxo_net* n, const float* x, int B, int P, int channel, int sigmoid, float* prob) {
    return fxo_net_forward_tiled(n, x, B, P, P, P, channel, sigmoid, prob);
}

/* ---- sliding window: src/ml/infer.hpp:456-864 (tta off, no crop, no checkpoint), per axis:
 * tile starts, Gaussian (sigma = tile / 8) and weight profile of each axis from its own extent -- */
int fxo_predict_tiled(const fxo_net* n, const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, int tz, int ty,
                      int tx, double overlap, int channel, int sigmoid, float* prob) {
    if (!fxo_net_tile_ok(n, tz, ty, tx)) return 1;
    int64_t zs[4096], ys[4096], xs[4096];
    const int64_t nz = fxo_tile_starts(dz, tz, overlap, zs, 4096), ny = fxo_tile_starts(dy, ty, overlap, ys, 4096),
                  nx = fxo_tile_starts(dx, tx, overlap, xs, 4096);
    if (nz > 4096 || ny > 4096 || nx > 4096) return 1;
    float* gz = (float*)malloc(sizeof(float) * (size_t)tz);
    float* gy = (float*)malloc(sizeof(float) * (size_t)ty);
    float* gx = (float*)malloc(sizeof(float) * (size_t)tx);
    fxo_gaussian1d(tz, gz);
    fxo_gaussian1d(ty, gy);
    fxo_gaussian1d(tx, gx);
    float* Wz = (float*)malloc(sizeof(float) * (size_t)dz);
    float* Wy = (float*)malloc(sizeof(float) * (size_t)dy);
    float* Wx = (float*)malloc(sizeof(float) * (size_t)dx);
    fxo_weight_profile(gz, tz, zs, nz, 0, dz, dz, Wz);
    fxo_weight_profile(gy, ty, ys, ny, 0, dy, dy, Wy);
    fxo_weight_profile(gx, tx, xs, nx, 0, dx, dx, Wx);
    const int64_t PN = (int64_t)tz * ty * tx;
    float* patch = (float*)malloc(sizeof(float) * (size_t)PN);
    float* sp = (float*)malloc(sizeof(float) * (size_t)PN);
    memset(prob, 0, sizeof(float) * (size_t)(dz * dy * dx));
    for (int64_t iz = 0; iz < nz; ++iz)
        for (int64_t iy = 0; iy < ny; ++iy)
            for (int64_t ix = 0; ix < nx; ++ix) {
                const int64_t z0 = zs[iz], y0 = ys[iy], x0 = xs[ix];
                fxo_fill_tile_u8(vol, dz, dy, dx, z0, y0, x0, tz, ty, tx, patch);
                fxo_norm_tile_zscore(patch, tz, ty, tx);
                fxo_net_forward_tiled(n, patch, 1, tz, ty, tx, channel, sigmoid, sp);
                /* scatter: prob += (gz*gy)*gx*p over the in-volume part (infer.hpp:631-653) */
#pragma omp parallel for
                for (int z = 0; z < tz; ++z) {
                    const int64_t oz = z0 + z;
                    if (oz >= dz) continue;
                    for (int y = 0; y < ty; ++y) {
                        const int64_t oy = y0 + y;
                        if (oy >= dy) break;
                        const float wzy = gz[z] * gy[y];
                        for (int x = 0; x < tx; ++x) {
                            const int64_t ox = x0 + x;
                            if (ox >= dx) break;
                            prob[(oz * dy + oy) * dx + ox] += wzy * gx[x] * sp[((int64_t)z * ty + y) * tx + x];
                        }
                    }
                }
            }
    /* normalize: v /= (Wz*Wy)*Wx where positive (infer.hpp:510-521) */
#pragma omp parallel for
    for (int64_t z = 0; z < dz; ++z)
        for (int64_t y = 0; y < dy; ++y) {
            const float wzy = Wz[z] * Wy[y];
            for (int64_t x = 0; x < dx; ++x) {
                const float w = wzy * Wx[x];
                if (w > 0.0f) prob[(z * dy + y) * dx + x] /= w;
            }
        }
    free(gz);
    free(gy);
    free(gx);
    free(Wz);
    free(Wy);
    free(Wx);
    free(patch);
    free(sp);
    return 0;
}

int fxo_predict_surface(const fxo_net* n, const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, int P,
                        double overlap, int channel, int sigmoid, float* prob) {
    if (P % 64 != 0) return 1;
    return fxo_predict_tiled(n, vol, dz, dy, dx, P, P, P, overlap, channel, sigmoid, prob);
}

/* u8 = (u8)(clamp(p, 0, 1) * 255 + 0.5): src/ml/inference.cpp:343-351 */
void fxo_prob_to_u8(const float* p, int64_t n, uint8_t* out) {
#pragma omp parallel for
    for (int64_t i = 0; i < n; ++i) {
        float v = p[i];
        v = v < 0.0f ? 0.0f : (v > 1.0f ? 1.0f : v);
        out[i] = (uint8_t)(v * 255.0f + 0.5f);
    }
}
