// net.cu — plain 3D UNet on the tcgen05 conv kernel + sliding-window driver (see net.cuh).
#include "net.cuh"
#include "pack.cuh"
#include "fenix_b200/ml/tiling.hpp"

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <cstdio>
#include <cstring>

namespace fxk {
cudaError_t launch_conv_tc(const ConvParams& p, int grid, size_t smem_bytes, cudaStream_t stream);
}

namespace fxh {

// Cycle counters of conv launches when the kernel is built with FX_CONV_TRACE (set by a trace
// driver through fx_conv_trace_buffer); null otherwise.
unsigned long long* g_conv_trace = nullptr;

using fenix::ml::gaussian1d;
using fenix::ml::tile_starts;

namespace {
constexpr float kE4M3Max = 448.f;
constexpr float kSlope = 0.01f;  // LeakyReLU negative slope (resenc_unet.hpp:49)
constexpr float kEps = 1e-5f;    // InstanceNorm3d eps (resenc_unet.hpp:44)

template <class T>
Status upload(T*& dst, const std::vector<T>& v, Net* /*unused*/, std::vector<void*>& allocs) {
    if (v.empty()) {
        dst = nullptr;
        return ok();
    }
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, v.size() * sizeof(T));
    if (e != cudaSuccess) return cuda_status(e, "cudaMalloc");
    allocs.push_back(p);
    e = cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_status(e, "cudaMemcpy");
    dst = static_cast<T*>(p);
    return ok();
}
}  // namespace

size_t DevProgram::smem() const {
    const size_t base = static_cast<size_t>(host.n_pipe) * host.stage_bytes + fxk::conv_tc_ctl_bytes() +
                        (fold ? fxk::conv_tc_fold_bytes(N_tile / 3) : 0);
    return zfold ? (base + 127) / 128 * 128 + host.bres_bytes : base;
}

Status cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return ok();
    return fail(kInternal, std::string(what) + ": " + cudaGetErrorString(e));
}

Net::~Net() {
    if (dev_ >= 0) cudaSetDevice(dev_);
    if (stream_) cudaStreamSynchronize(stream_);
    for (void* p : allocs_) cudaFree(p);
    if (stream_) cudaStreamDestroy(stream_);
}

void* Net::dalloc(size_t bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
    allocs_.push_back(p);
    return p;
}

// ---- weights -> layer plans ------------------------------------------------------------------
Status Net::parse(const WeightMap& wm) {
    auto get = [&](const std::string& n) -> const HostTensor* {
        auto it = wm.find(n);
        return it == wm.end() ? nullptr : &it->second;
    };
    // residual-encoder checkpoints: {encoder|shared_encoder}.stem + stages.{s}.blocks.{b}
    if (get("encoder.stem.convs.0.conv.weight")) return parse_resenc(wm, "encoder", "decoder");
    if (get("shared_encoder.stem.convs.0.conv.weight")) {
        // task_decoders.<task>: the one task holding seg_layers
        for (const auto& kv : wm) {
            const std::string& n = kv.first;
            const std::string pre = "task_decoders.";
            const size_t k = n.find(".seg_layers.");
            if (n.rfind(pre, 0) == 0 && k != std::string::npos) return parse_resenc(wm, "shared_encoder", n.substr(0, k));
        }
        // the ink checkpoints: shared_decoder.* without seg_layers + task_heads.<task> (one 1x1x1
        // conv, src/ml/nets/resenc_unet.hpp:291-316)
        if (get("shared_decoder.transpconvs.0.weight"))
            for (const auto& kv : wm) {
                const std::string& n = kv.first;
                const std::string pre = "task_heads.";
                if (n.rfind(pre, 0) == 0 && n.size() > 7 && n.compare(n.size() - 7, 7, ".weight") == 0)
                    return parse_resenc(wm, "shared_encoder", "shared_decoder", n.substr(0, n.size() - 7));
            }
        return fail(kUnsupported, "fxweights: residual encoder without task_decoders.<task>.seg_layers or task_heads.<task>");
    }
    // encoder.stages.{s}.convs.{i}.conv.weight
    S_ = 0;
    while (get("encoder.stages." + std::to_string(S_) + ".convs.0.conv.weight")) ++S_;
    if (S_ < 2) return fail(kDecode, "fxweights: expected >= 2 encoder stages (encoder.stages.{s}.convs.{i}.conv.weight)");
    nconv_ = 0;
    while (get("encoder.stages.0.convs." + std::to_string(nconv_) + ".conv.weight")) ++nconv_;
    if (nconv_ < 1) return fail(kDecode, "fxweights: no convs in encoder stage 0");
    F_.clear();
    // the axes each stage halves, read from the transposed conv that undoes it: its kernel is 2 along
    // the halved axes and 1 along the others (nnU-Net's per-stage strides, e.g. (1, 2, 2))
    smask_.assign(S_, 0);
    for (int s = 1; s < S_; ++s) {
        const std::string tp = "decoder.transpconvs." + std::to_string(S_ - 1 - s);
        const HostTensor* w = get(tp + ".weight");
        if (!w || w->shape.size() != 5) return fail(kDecode, "fxweights: missing or malformed " + tp + ".weight");
        int m = 0;
        for (int a = 0; a < 3; ++a) {
            const int64_t k = w->shape[2 + a];
            if (k != 1 && k != 2) return fail(kUnsupported, "fxweights: " + tp + " kernel must be 1 or 2 along each axis");
            if (k == 2) m |= 4 >> a;
        }
        if (!m) return fail(kUnsupported, "fxweights: " + tp + " does not upsample");
        smask_[s] = m;
    }
    auto conv_layer = [&](const std::string& pre, Layer& L) -> Status {
        const HostTensor* w = get(pre + ".conv.weight");
        const HostTensor* g = get(pre + ".norm.weight");
        const HostTensor* b = get(pre + ".norm.bias");
        if (!w || !g || !b) return fail(kDecode, "fxweights: missing " + pre + ".{conv.weight,norm.weight,norm.bias}");
        if (w->shape.size() != 5 || w->shape[2] != 3 || w->shape[3] != 3 || w->shape[4] != 3)
            return fail(kUnsupported, "fxweights: " + pre + " must be a 3x3x3 conv");
        L.Cout = static_cast<int>(w->shape[0]);
        L.Cin = static_cast<int>(w->shape[1]);
        L.w = w->data;
        L.gamma = g->data;
        L.beta = b->data;
        L.name = pre;
        return ok();
    };
    enc_.assign(static_cast<size_t>(S_) * nconv_, Layer{});
    int prev = 1;
    for (int s = 0; s < S_; ++s)
        for (int i = 0; i < nconv_; ++i) {
            Layer& L = enc_[s * nconv_ + i];
            Status st = conv_layer("encoder.stages." + std::to_string(s) + ".convs." + std::to_string(i), L);
            if (!st.ok()) return st;
            if (L.Cin != (i == 0 ? prev : L.Cout)) return fail(kDecode, "fxweights: channel mismatch at " + L.name);
            L.stride = (i == 0 && s > 0) ? 2 : 1;
            L.smask = (i == 0 && s > 0) ? smask_[s] : 0;
            L.kind = (s == 0 && i == 0) ? Layer::kFirst : Layer::kConv;
            L.lin = (i == 0 && s > 0) ? s - 1 : s;
            L.lout = s;
            if (i == 0) F_.push_back(L.Cout);
            prev = L.Cout;
        }
    if (F_[0] < 1 || enc_[0].Cin != 1) return fail(kUnsupported, "net: the first conv must take 1 input channel");
    up_.assign(S_ - 1, Layer{});
    dec_.assign(static_cast<size_t>(S_ - 1) * nconv_, Layer{});
    for (int t = 0; t < S_ - 1; ++t) {
        const int lvl = S_ - 2 - t;
        const std::string tp = "decoder.transpconvs." + std::to_string(t);
        const HostTensor* w = get(tp + ".weight");
        const HostTensor* b = get(tp + ".bias");
        if (!w || !b) return fail(kDecode, "fxweights: missing " + tp + ".{weight,bias}");
        Layer& U = up_[lvl];  // kernel shape already checked against the stage's mask above
        U.kind = Layer::kUp;
        U.name = tp;
        U.Cin = static_cast<int>(w->shape[0]);
        U.Cout = static_cast<int>(w->shape[1]);
        if (U.Cin != F_[lvl + 1] || U.Cout != F_[lvl]) return fail(kDecode, "fxweights: channel mismatch at " + tp);
        U.w = w->data;
        U.b = b->data;
        U.stride = 2;
        U.smask = smask_[lvl + 1];
        U.lin = lvl + 1;
        U.lout = lvl;
        for (int i = 0; i < nconv_; ++i) {
            Layer& L = dec_[lvl * nconv_ + i];
            Status st = conv_layer("decoder.stages." + std::to_string(t) + ".convs." + std::to_string(i), L);
            if (!st.ok()) return st;
            if (L.Cout != F_[lvl] || L.Cin != (i == 0 ? 2 * F_[lvl] : F_[lvl]))
                return fail(kDecode, "fxweights: channel mismatch at " + L.name);
            L.lin = L.lout = lvl;
        }
    }
    const std::string sl = "decoder.seg_layers." + std::to_string(S_ - 2);
    const HostTensor* hw = get(sl + ".weight");
    const HostTensor* hb = get(sl + ".bias");
    if (!hw || !hb) return fail(kDecode, "fxweights: missing " + sl + ".{weight,bias}");
    ncls_ = static_cast<int>(hw->shape[0]);
    if (hw->shape[1] != F_[0] || ncls_ < 1 || ncls_ > 2) return fail(kUnsupported, "net: head must map F0 -> 1 or 2 classes");
    head_w_ = hw->data;
    head_b_ = hb->data;
    return ok();
}

// Residual-encoder UNet (nets::ResEncUNet, src/ml/nets/resenc_unet.hpp:159-318): stem ConvStack
// (1 conv), stages of BasicBlockD (conv1 with the stage's stride, conv2 without activation,
// optional scSE, skip = [AvgPool(2)] + [1x1 conv + norm], add, LeakyReLU), and the plain decoder
// (transpconvs, one ConvStack per stage, seg_layers) under `dec`.
Status Net::parse_resenc(const WeightMap& wm, const std::string& enc, const std::string& dec, const std::string& head) {
    auto get = [&](const std::string& n) -> const HostTensor* {
        auto it = wm.find(n);
        return it == wm.end() ? nullptr : &it->second;
    };
    auto conv_layer = [&](const std::string& pre, Layer& L, int k) -> Status {
        const HostTensor* w = get(pre + ".conv.weight");
        const HostTensor* g = get(pre + ".norm.weight");
        const HostTensor* b = get(pre + ".norm.bias");
        if (!w || !g || !b) return fail(kDecode, "fxweights: missing " + pre + ".{conv.weight,norm.weight,norm.bias}");
        if (w->shape.size() != 5 || w->shape[2] != k || w->shape[3] != k || w->shape[4] != k)
            return fail(kUnsupported, "fxweights: " + pre + " must be a " + std::to_string(k) + "^3 conv");
        L.Cout = static_cast<int>(w->shape[0]);
        L.Cin = static_cast<int>(w->shape[1]);
        L.w = w->data;
        L.gamma = g->data;
        L.beta = b->data;
        L.name = pre;
        return ok();
    };
    resenc_ = true;
    enc_.clear();
    smask_.clear();
    blocks_.clear();
    F_.clear();
    Layer stem;
    Status st = conv_layer(enc + ".stem.convs.0", stem, 3);
    if (!st.ok()) return st;
    if (stem.Cin != 1) return fail(kUnsupported, "net: the stem must take 1 input channel");
    stem.kind = Layer::kFirst;
    stem.stride = 1;
    stem.lin = stem.lout = 0;
    enc_.push_back(stem);
    S_ = 0;
    while (get(enc + ".stages." + std::to_string(S_) + ".blocks.0.conv1.conv.weight")) ++S_;
    if (S_ < 2) return fail(kDecode, "fxweights: expected >= 2 residual stages");
    if (S_ > 16) return fail(kUnsupported, "net: more than 16 stages");
    int prev = stem.Cout;
    int slot = 5 * S_;
    for (int s = 0; s < S_; ++s) {
        for (int b = 0;; ++b) {
            const std::string pre = enc + ".stages." + std::to_string(s) + ".blocks." + std::to_string(b);
            if (!get(pre + ".conv1.conv.weight")) {
                if (b == 0) return fail(kDecode, "fxweights: empty stage " + std::to_string(s));
                break;
            }
            ResBlock K;
            K.stage = s;
            K.stride = (b == 0 && s > 0) ? 2 : 1;
            Layer c1, c2;
            if ((st = conv_layer(pre + ".conv1", c1, 3)).code || (st = conv_layer(pre + ".conv2", c2, 3)).code) return st;
            if (c1.Cin != (b == 0 ? prev : c1.Cout) || c2.Cin != c1.Cout || c2.Cout != c1.Cout)
                return fail(kDecode, "fxweights: channel mismatch at " + pre);
            c1.kind = c2.kind = Layer::kConv;
            c1.stride = K.stride;
            c1.smask = K.stride == 2 ? 7 : 0;
            c2.stride = 1;
            c1.lin = K.stride == 2 ? s - 1 : s;
            c1.lout = c2.lin = c2.lout = s;
            K.c1 = static_cast<int>(enc_.size());
            enc_.push_back(c1);
            K.c2 = static_cast<int>(enc_.size());
            enc_.push_back(c2);
            const std::string pj = pre + ".skip." + std::to_string(K.stride == 2 ? 1 : 0);
            if (c1.Cin != c1.Cout) {
                Layer pl;
                if ((st = conv_layer(pj, pl, 1)).code) return st;
                pl.kind = Layer::kProj;
                pl.stride = K.stride;
                pl.smask = K.stride == 2 ? 7 : 0;
                pl.lin = c1.lin;
                pl.lout = s;
                K.proj = static_cast<int>(enc_.size());
                enc_.push_back(pl);
            } else {
                K.avgpool = K.stride == 2;
            }
            const std::string se = pre + ".squeeze_excitation.";
            if (get(se + "sSE.conv.weight")) {
                const HostTensor *f1w = get(se + "cSE.fc1.weight"), *f1b = get(se + "cSE.fc1.bias"),
                                 *f2w = get(se + "cSE.fc2.weight"), *f2b = get(se + "cSE.fc2.bias"),
                                 *sw = get(se + "sSE.conv.weight"), *sb = get(se + "sSE.conv.bias");
                const int C = c2.Cout;
                if (!f1w || !f1b || !f2w || !f2b || !sb || f1w->shape.size() != 5 || f1w->shape[1] != C ||
                    f2w->shape[0] != C || sw->shape[1] != C)
                    return fail(kDecode, "fxweights: malformed " + se + "*");
                const int rd = static_cast<int>(f1w->shape[0]);
                K.se = true;
                // GAP of IN(conv2) (no activation) is the norm's bias: the cSE gate is a constant
                std::vector<float> hid(rd);
                for (int r = 0; r < rd; ++r) {
                    double a = f1b->data[r];
                    for (int c = 0; c < C; ++c) a += static_cast<double>(f1w->data[static_cast<size_t>(r) * C + c]) * c2.beta[c];
                    hid[r] = a > 0.0 ? static_cast<float>(a) : 0.f;
                }
                K.cgate.resize(C);
                for (int c = 0; c < C; ++c) {
                    double a = f2b->data[c];
                    for (int r = 0; r < rd; ++r) a += static_cast<double>(f2w->data[static_cast<size_t>(c) * rd + r]) * hid[r];
                    K.cgate[c] = static_cast<float>(1.0 / (1.0 + std::exp(-a)));
                }
                K.sse_w.assign(sw->data.begin(), sw->data.begin() + C);
                K.sse_b = sb->data[0];
            }
            K.slot_x = slot++;
            K.slot_h = slot++;
            blocks_.push_back(std::move(K));
            prev = c1.Cout;
        }
        F_.push_back(prev);
        smask_.push_back(s > 0 ? 7 : 0);
    }
    nslots_ = slot + 1;  // + the last stage's output (the first transposed conv's input)
    // decoder: transpconvs, one or more convs per stage, seg_layers (as the plain decoder)
    nconv_ = 0;
    while (get(dec + ".stages.0.convs." + std::to_string(nconv_) + ".conv.weight")) ++nconv_;
    if (nconv_ < 1) return fail(kDecode, "fxweights: no convs in " + dec + ".stages.0");
    up_.assign(S_ - 1, Layer{});
    dec_.assign(static_cast<size_t>(S_ - 1) * nconv_, Layer{});
    for (int t = 0; t < S_ - 1; ++t) {
        const int lvl = S_ - 2 - t;
        const std::string tp = dec + ".transpconvs." + std::to_string(t);
        const HostTensor* w = get(tp + ".weight");
        const HostTensor* b = get(tp + ".bias");
        if (!w || !b) return fail(kDecode, "fxweights: missing " + tp + ".{weight,bias}");
        Layer& U = up_[lvl];  // kernel shape already checked against the stage's mask above
        U.kind = Layer::kUp;
        U.name = tp;
        U.Cin = static_cast<int>(w->shape[0]);
        U.Cout = static_cast<int>(w->shape[1]);
        if (U.Cin != F_[lvl + 1] || U.Cout != F_[lvl]) return fail(kDecode, "fxweights: channel mismatch at " + tp);
        U.w = w->data;
        U.b = b->data;
        U.stride = 2;
        U.smask = 7;
        U.lin = lvl + 1;
        U.lout = lvl;
        for (int i = 0; i < nconv_; ++i) {
            Layer& L = dec_[lvl * nconv_ + i];
            if ((st = conv_layer(dec + ".stages." + std::to_string(t) + ".convs." + std::to_string(i), L, 3)).code)
                return st;
            if (L.Cout != F_[lvl] || L.Cin != (i == 0 ? 2 * F_[lvl] : F_[lvl]))
                return fail(kDecode, "fxweights: channel mismatch at " + L.name);
            L.lin = L.lout = lvl;
        }
    }
    // the head: the deepest decoder stage's seg_layers, or a separate task head (ink checkpoints)
    const std::string sl = head.empty() ? dec + ".seg_layers." + std::to_string(S_ - 2) : head;
    const HostTensor* hw = get(sl + ".weight");
    const HostTensor* hb = get(sl + ".bias");
    if (!hw || !hb) return fail(kDecode, "fxweights: missing " + sl + ".{weight,bias}");
    ncls_ = static_cast<int>(hw->shape[0]);
    if (hw->shape.size() != 5 || hw->shape[1] != F_[0] || ncls_ < 1 || ncls_ > 2)
        return fail(kUnsupported, "net: head must map F0 -> 1 or 2 classes");
    head_w_ = hw->data;
    head_b_ = hb->data;
    return ok();
}

// ---- layer program construction -------------------------------------------------------------
// The x-tap fold (A collector shared by the three x taps) is off unless FENIX_B200_CONV_FOLD=1:
// its MMAs run 1.6x faster, but its epilogue (three accumulators and a cross-lane row shift)
// costs more than it saves with the current epilogue, measured on the 32- and 64-channel layers.
// Read whenever a program is built, so one process can run and compare both programs.
static bool fold_enabled() {
    const char* v = std::getenv("FENIX_B200_CONV_FOLD");
    return v && v[0] == '1';
}

// z-plane fold (fxk::ConvParams::zfold) for 3x3x3 stride-1 convs of at most 64 output channels
// whose weights fit in shared memory next to three stages; FENIX_B200_CONV_ZFOLD=0 turns it off.
static bool zfold_enabled() {
    const char* v = std::getenv("FENIX_B200_CONV_ZFOLD");
    return !(v && v[0] == '0');
}

Status build_layer_program(Layer& L, int q, ActGeom gin, ActGeom gout, int Bmax, int sm_count,
                           std::vector<void*>& allocs_) {
    DevProgram& dp = L.prog[q];
    ProgramSpec sp;
    const bool fp8 = q == 1;
    sp.optype = q;
    sp.elem = fp8 ? 1 : 2;
    sp.cg = fp8 ? 16 : 8;
    const int Bmax_ = Bmax, sm_count_ = sm_count;
    Net* this_net = nullptr;
    if (fp8 && L.wscale.empty()) {
        // per-output-channel weight scale amax/448 (tools/ml-export/fp8_conv3d_op.py:1494-1504)
        L.wscale.assign(L.Cout, 1.f);
        if (L.kind == Layer::kUp) {
            for (int co = 0; co < L.Cout; ++co) {
                float m = 0.f;
                const int nph = 1 << __builtin_popcount(static_cast<unsigned>(L.smask));
                for (int ci = 0; ci < L.Cin; ++ci)
                    for (int a = 0; a < nph; ++a)
                        m = std::max(m, std::fabs(L.w[(static_cast<size_t>(ci) * L.Cout + co) * nph + a]));
                L.wscale[co] = std::max(m, 1e-8f) / kE4M3Max;
            }
        } else {
            const size_t per = static_cast<size_t>(L.Cin) * (L.kind == Layer::kProj ? 1 : 27);
            for (int co = 0; co < L.Cout; ++co) {
                float m = 0.f;
                for (size_t k = 0; k < per; ++k) m = std::max(m, std::fabs(L.w[co * per + k]));
                L.wscale[co] = std::max(m, 1e-8f) / kE4M3Max;
            }
        }
    }
    std::vector<float> colscale, ratio;
    dp.acc_scale = 1.f;
    bool fold = false;
    if (L.kind == Layer::kFirst) {
        // One input channel: a cell carries the three x taps of a voxel, and the value is split into
        // two 16-bit terms (first_layer_cells): group 0 = [hi x3, lo x3] times the 16-bit weights,
        // group 1 = [hi x3] times the weights' rounding residues, so the first conv sees its input
        // and weights to about twice the 16-bit precision. One MMA (K = both groups) per (kz, ky).
        if (fp8) return fail(kInternal, "first layer runs with 16-bit operands");
        sp.G = 2;
        const ActGeom g = gout;
        const int64_t Wp = g.W + 2, P2 = static_cast<int64_t>(g.H + 2) * Wp;
        for (int kz = 0; kz < 3; ++kz)
            for (int ky = 0; ky < 3; ++ky) sp.taps.push_back({0, (kz - 1) * P2 + (ky - 1) * Wp, kz * 3 + ky, kz});
        const Layer* Lp = &L;
        const int q16 = q;
        sp.wval = [Lp, q16](int n, int ci, int wk) {
            const int grp = ci / 8, j = ci % 8;
            const int kx = grp == 0 ? (j < 3 ? j : (j < 6 ? j - 3 : -1)) : (j < 3 ? j : -1);
            if (kx < 0) return 0.f;
            const float w = Lp->w[static_cast<size_t>(n) * 27 + wk * 3 + kx];
            return grp == 0 ? w : w - round16_host(w, q16);
        };
        sp.N_total = L.Cout;
        dp.rowspace = gout;
    } else if (L.kind == Layer::kConv) {
        if (L.Cin % sp.cg) return fail(kUnsupported, L.name + ": input channels must be a multiple of " + std::to_string(sp.cg));
        sp.G = L.Cin / sp.cg;
        fold = L.stride == 1 && (L.Cout == 16 || L.Cout == 32 || L.Cout == 64) && fold_enabled();
        if (fold) {
            // x-tap fold: 9 (kz, ky) taps whose A tile starts one row early; B column n holds x tap
            // n / Cout of output channel n % Cout
            const int64_t Wp = gin.W + 2, P2 = static_cast<int64_t>(gin.H + 2) * Wp;
            for (int kz = 0; kz < 3; ++kz)
                for (int ky = 0; ky < 3; ++ky) sp.taps.push_back({0, (kz - 1) * P2 + (ky - 1) * Wp - 1, kz * 9 + ky * 3, kz});
        } else if (L.stride == 1) {
            const int64_t Wp = gin.W + 2, P2 = static_cast<int64_t>(gin.H + 2) * Wp;
            for (int kz = 0; kz < 3; ++kz)
                for (int ky = 0; ky < 3; ++ky)
                    for (int kx = 0; kx < 3; ++kx)
                        sp.taps.push_back({0, (kz - 1) * P2 + (ky - 1) * Wp + (kx - 1), kz * 9 + ky * 3 + kx, kz});
            const int64_t bres = 27LL * (sp.G / 2) * L.Cout * 32;
            if (zfold_enabled() && L.Cout <= 64 && sp.G % 2 == 0 && bres <= 112 * 1024 && gin.D >= 2) {
                sp.zfold = true;
                sp.zWp = Wp;
                sp.zP2 = P2;
            }
        } else {
            // stride 2 along the axes of smask: the input is the phase-split copy (one sub-volume per
            // parity of the halved axes, each on the output grid); a tap on a halved axis picks the
            // phase of its parity and shifts by k / 2 - 1, on a full axis it shifts by k - 1
            const int64_t Wp = gout.W + 2, P2 = static_cast<int64_t>(gout.H + 2) * Wp;
            const int m = L.smask;
            for (int kz = 0; kz < 3; ++kz)
                for (int ky = 0; ky < 3; ++ky)
                    for (int kx = 0; kx < 3; ++kx) {
                        int phi = 0;
                        int64_t off = 0;
                        const int k[3] = {kz, ky, kx};
                        const int64_t step[3] = {P2, Wp, 1};
                        for (int a = 0; a < 3; ++a) {
                            if (m & (4 >> a)) {
                                phi = (phi << 1) | (k[a] & 1);
                                off += (k[a] / 2 - 1) * step[a];
                            } else {
                                off += (k[a] - 1) * step[a];
                            }
                        }
                        const int zkey = (m & 4) ? kz / 2 : kz;  // taps of one z shift share a window
                        sp.taps.push_back({phi, off, kz * 9 + ky * 3 + kx, phi * 3 + zkey});
                    }
        }
        const Layer* Lp = &L;
        const bool f8 = fp8;
        const int fc = fold ? L.Cout : 0;
        sp.wval = [Lp, f8, fc](int n, int ci, int wk) {
            if (ci >= Lp->Cin) return 0.f;
            const int co = fc ? n % fc : n, kx = fc ? n / fc : 0;  // fold: wk is kz*9 + ky*3
            const float v = Lp->w[(static_cast<size_t>(co) * Lp->Cin + ci) * 27 + wk + kx];
            return f8 ? v / Lp->wscale[co] : v;
        };
        sp.N_total = fold ? 3 * L.Cout : L.Cout;
        dp.rowspace = gout;
        if (fp8) {
            colscale.resize(L.Cout);
            for (int co = 0; co < L.Cout; ++co) colscale[co] = L.in_scale * L.wscale[co];
            // one epilogue factor = the largest channel's, so stored f16 values are never larger
            // than that channel's own range; the per-channel remainder (<= 1) goes to the stats
            dp.acc_scale = *std::max_element(colscale.begin(), colscale.end());
            ratio.resize(L.Cout);
            for (int co = 0; co < L.Cout; ++co) ratio[co] = colscale[co] / dp.acc_scale;
        }
    } else if (L.kind == Layer::kProj) {
        // 1x1x1 projection; with stride 2 the AvgPool(2) in front of it makes it a 2x2x2 stride-2
        // conv with weights / 8: taps (kz, ky, kx) in {1, 2}^3 of the stride-2 tap scheme
        if (L.Cin % sp.cg) return fail(kUnsupported, L.name + ": input channels must be a multiple of " + std::to_string(sp.cg));
        sp.G = L.Cin / sp.cg;
        float wmul = 1.f;
        if (L.stride == 1) {
            sp.taps.push_back({0, 0, 0, 0});
        } else {
            wmul = 0.125f;
            const int64_t Wp = gout.W + 2, P2 = static_cast<int64_t>(gout.H + 2) * Wp;
            for (int kz = 1; kz < 3; ++kz)
                for (int ky = 1; ky < 3; ++ky)
                    for (int kx = 1; kx < 3; ++kx) {
                        const int phi = ((kz & 1) << 2) | ((ky & 1) << 1) | (kx & 1);
                        const int64_t off = (kz / 2 - 1) * P2 + (ky / 2 - 1) * Wp + (kx / 2 - 1);
                        sp.taps.push_back({phi, off, 0, phi});
                    }
        }
        const Layer* Lp = &L;
        const bool f8 = fp8;
        sp.wval = [Lp, f8, wmul](int n, int ci, int) {
            if (ci >= Lp->Cin) return 0.f;
            const float v = Lp->w[static_cast<size_t>(n) * Lp->Cin + ci] * wmul;
            return f8 ? v / (Lp->wscale[n] * wmul) : v;
        };
        sp.N_total = L.Cout;
        dp.rowspace = gout;
        if (fp8) {
            colscale.resize(L.Cout);
            for (int co = 0; co < L.Cout; ++co) colscale[co] = L.in_scale * L.wscale[co] * wmul;
            dp.acc_scale = *std::max_element(colscale.begin(), colscale.end());
            ratio.resize(L.Cout);
            for (int co = 0; co < L.Cout; ++co) ratio[co] = colscale[co] / dp.acc_scale;
        }
    } else {  // kUp
        if (L.Cin % sp.cg) return fail(kUnsupported, L.name + ": input channels must be a multiple of " + std::to_string(sp.cg));
        sp.G = L.Cin / sp.cg;
        sp.taps.push_back({0, 0, 0, 0});
        const Layer* Lp = &L;
        const bool f8 = fp8;
        // one output phase per kernel position: weights [Cin][Cout][kz][ky][kx], 2 along the axes of
        // smask and 1 along the others, so the positions are the phases in z, y, x bit order
        const int nph = 1 << __builtin_popcount(static_cast<unsigned>(L.smask));
        sp.wval = [Lp, f8, nph](int n, int ci, int) {
            if (ci >= Lp->Cin) return 0.f;
            const int co = n % Lp->Cout, a = n / Lp->Cout;
            const float v = Lp->w[(static_cast<size_t>(ci) * Lp->Cout + co) * nph + a];
            return f8 ? v / Lp->wscale[co] : v;
        };
        sp.N_total = nph * L.Cout;
        dp.rowspace = gin;
        if (fp8) {
            colscale.resize(L.Cout);
            for (int co = 0; co < L.Cout; ++co) colscale[co] = L.in_scale * L.wscale[co];
        }
    }
    // tiling of N and M
    const int N_total = sp.N_total;
    if (sp.zfold) {  // one N tile; 2 segments x Z planes (Z 4 at N 32, 2 at N 64); 2 TMEM slots
        const ActGeom& g = gout;
        const int S = 2, Zp = N_total <= 32 ? 4 : 2, R = S * Zp;
        const int64_t Wp = g.W + 2, P2 = static_cast<int64_t>(g.H + 2) * Wp;
        const int zseg = static_cast<int>((P2 - 2 * (Wp + 1) + 128 * S - 1) / (128 * S));
        sp.N_tile = N_total;
        sp.R = Zp;
        sp.zsegs = S;
        sp.block_rows = 128;
        Program zp;
        std::string zerr = build_program(sp, zp);
        if (zerr.empty()) {
            dp.host = std::move(zp);
            dp.R = R;
            dp.N_tile = N_total;
            dp.acc_slots = 2;
            uint32_t cols = 32;
            while (cols < static_cast<uint32_t>(2 * R * N_total)) cols <<= 1;
            dp.tmem_cols = cols;
            dp.zseg = zseg;
            dp.zplanes = Zp;
            dp.n_units_m = static_cast<int>((g.D + Zp - 1) / Zp) * zseg;
            dp.zfold = true;
            dp.fold = false;
            dp.block_rows = 128;
            dp.optype = q;
            Status zst;
            if ((zst = upload(dp.wpack, dp.host.wpack, this_net, allocs_)).code) return zst;
            if ((zst = upload(dp.colscale, colscale, this_net, allocs_)).code) return zst;
            if ((zst = upload(dp.ratio, ratio, this_net, allocs_)).code) return zst;
            dp.built = true;
            return ok();
        }
        sp.zfold = false;  // weights do not fit next to three stages: the regular program
    }
    int N_tile = N_total <= 256 ? N_total : (N_total == 320 ? 320 : 256);
    // A stride-2 conv 256 columns wide runs as two 128-column tiles: its phase-split windows hold
    // few taps each, so halving the B block per K step doubles the groups per stage and the units
    // (the 16^3 encoder conv of the surface net: 5.43 -> 3.62 ms per 343 tiles of 128^3; the
    // stride-1 256-column layers measured no gain, and 64-column tiles lost).
    if (L.kind == Layer::kConv && L.stride == 2 && N_total == 256) N_tile = 128;
    if (N_total % N_tile) return fail(kUnsupported, L.name + ": output width " + std::to_string(N_total) + " not tileable");
    int R = N_tile <= 32 ? 8 : (N_tile <= 64 ? 4 : (N_tile <= 128 ? 2 : 1));
    const int brows = fold ? 126 : 128;
    if (fold) R = N_tile <= 48 ? 4 : (N_tile <= 96 ? 2 : 1);  // two slots of R x 3 Cout columns in 512
    const ActGeom& rs = dp.rowspace;
    const int64_t rows = static_cast<int64_t>(rs.D) * (rs.H + 2) * (rs.W + 2);
    auto units = [&](int r) { return ((rows + brows * r - 1) / (brows * r)) * Bmax_ * (N_total / N_tile); };
    while (R > 1 && units(R) < 2 * sm_count_) R /= 2;
    const int slots = R * N_tile <= 256 ? 2 : 1;
    uint32_t cols = 32;
    while (cols < static_cast<uint32_t>(slots * R * N_tile)) cols <<= 1;
    if (cols > 512) return fail(kInternal, L.name + ": accumulator does not fit in TMEM");
    sp.N_tile = N_tile;
    sp.R = R;
    sp.block_rows = brows;
    if (fold) sp.smem_total -= static_cast<int>(fxk::conv_tc_fold_bytes(L.Cout));
    Status st;
    {
        std::string err = build_program(sp, dp.host);
        if (!err.empty()) return fail(kInternal, L.name + ": " + err);
    }
    dp.R = R;
    dp.N_tile = N_tile;
    dp.acc_slots = slots;
    dp.tmem_cols = cols;
    dp.n_units_m = static_cast<int>((rows + static_cast<int64_t>(brows) * R - 1) / (static_cast<int64_t>(brows) * R));
    dp.fold = fold;
    dp.block_rows = brows;
    dp.optype = q;
    if ((st = upload(dp.wpack, dp.host.wpack, this_net, allocs_)).code) return st;
    if ((st = upload(dp.colscale, colscale, this_net, allocs_)).code) return st;
    if ((st = upload(dp.ratio, ratio, this_net, allocs_)).code) return st;
    if (L.kind == Layer::kUp && (st = upload(dp.bias, L.b, this_net, allocs_)).code) return st;
    dp.built = true;
    return ok();
}

Status Net::build_layer(Layer& L, int q) {
    Status st = build_layer_program(L, q, level(L.lin), level(L.lout), Bmax_, sm_count_, allocs_);
    if (!st.ok()) return st;
    // statistics buffers (shared by both precisions): one record per 128-row block and warp
    if (L.kind != Layer::kUp && !L.d_partials) {
        const ActGeom g = level(L.lout);
        const int64_t rows = static_cast<int64_t>(g.D) * (g.H + 2) * (g.W + 2);
        const int64_t nrec_max = std::max<int64_t>(((rows + 125) / 126), sm_count_) * fxk::kStatRecsPerUnit;
        L.d_partials = static_cast<float*>(dalloc(sizeof(float) * Bmax_ * nrec_max * L.Cout * 2));
        L.nrec_cap = nrec_max;
        if (L.d_partials) cudaMemset(L.d_partials, 0, sizeof(float) * Bmax_ * nrec_max * L.Cout * 2);
        L.d_ss = static_cast<float*>(dalloc(sizeof(float) * Bmax_ * L.Cout * 2));
        if (!L.d_partials || !L.d_ss) return fail(kInternal, "cudaMalloc: stats buffers");
        if ((st = upload(L.d_gamma, L.gamma, this, allocs_)).code) return st;
        if ((st = upload(L.d_beta, L.beta, this, allocs_)).code) return st;
    }
    return ok();
}

Status Net::alloc() {
    const ActGeom g0 = level(0);
    // the first conv's input: two 16-bit groups per voxel (the value as hi + lo, first_layer_cells)
    l0_ = static_cast<uint8_t*>(dalloc(static_cast<size_t>(Bmax_) * 2 * g0.gs()));
    if (!l0_) return fail(kInternal, "cudaMalloc: first-layer input");
    cudaMemset(l0_, 0, static_cast<size_t>(Bmax_) * 2 * g0.gs());
    pn_.assign(S_, nullptr);
    act_.assign(S_, nullptr);
    cat_.assign(S_, nullptr);
    ph_.assign(S_, nullptr);
    for (int s = 0; s < S_; ++s) {
        const ActGeom g = level(s);
        const size_t bytes = static_cast<size_t>(Bmax_) * (F_[s] / 8) * g.gs();
        pn_[s] = static_cast<uint8_t*>(dalloc(bytes));
        act_[s] = static_cast<uint8_t*>(dalloc(bytes));
        if (!pn_[s] || !act_[s]) return fail(kInternal, "cudaMalloc: activations");
        cudaMemset(act_[s], 0, bytes);
        if (s < S_ - 1) {
            cat_[s] = static_cast<uint8_t*>(dalloc(2 * bytes));
            const ActGeom gn = level(s + 1);
            const int nph = 1 << __builtin_popcount(static_cast<unsigned>(smask_[s + 1]));
            const size_t pbytes = static_cast<size_t>(Bmax_) * (F_[s] / 8) * nph * gn.gs();
            ph_[s] = static_cast<uint8_t*>(dalloc(pbytes));
            if (!cat_[s] || !ph_[s]) return fail(kInternal, "cudaMalloc: skip buffers");
            cudaMemset(cat_[s], 0, 2 * bytes);
            cudaMemset(ph_[s], 0, pbytes);
        }
    }
    if (resenc_) {
        h_.assign(S_, nullptr);
        xf_.assign(S_, nullptr);
        pnx_.assign(S_, nullptr);
        res_.assign(S_, nullptr);
        sg_.assign(S_, nullptr);
        for (int s = 0; s < S_; ++s) {
            const ActGeom g = level(s);
            const size_t bytes = static_cast<size_t>(Bmax_) * (F_[s] / 8) * g.gs();
            bool proj = false, pool = false, se = false;
            for (const ResBlock& K : blocks_)
                if (K.stage == s) {
                    proj |= K.proj >= 0;
                    pool |= K.avgpool;
                    se |= K.se;
                }
            for (uint8_t** p : {&h_[s], &xf_[s]}) {
                *p = static_cast<uint8_t*>(dalloc(bytes));
                if (!*p) return fail(kInternal, "cudaMalloc: residual buffers");
                cudaMemset(*p, 0, bytes);
            }
            if (proj && !(pnx_[s] = static_cast<uint8_t*>(dalloc(bytes)))) return fail(kInternal, "cudaMalloc: projection");
            if (pool && !(res_[s] = static_cast<uint8_t*>(dalloc(bytes)))) return fail(kInternal, "cudaMalloc: pooled residual");
            if (se && !(sg_[s] = static_cast<float*>(dalloc(sizeof(float) * Bmax_ * g.D * g.H * g.W))))
                return fail(kInternal, "cudaMalloc: sSE gate");
        }
        for (ResBlock& K : blocks_) {
            if (!K.se) continue;
            Status st = upload(K.d_cgate, K.cgate, this, allocs_);
            if (st.ok()) st = upload(K.d_sse_w, K.sse_w, this, allocs_);
            if (!st.ok()) return st;
        }
    }
    nslots_ = std::max(nslots_, 5 * S_);
    d_sums_ = static_cast<unsigned long long*>(dalloc(sizeof(unsigned long long) * 2 * Bmax_));
    d_hist_ = static_cast<unsigned*>(dalloc(sizeof(unsigned) * 256 * Bmax_));
    d_luts_ = static_cast<float*>(dalloc(sizeof(float) * 256 * Bmax_));
    if (!d_hist_ || !d_luts_) return fail(kInternal, "cudaMalloc: normalisation tables");
    d_amax_ = static_cast<unsigned*>(dalloc(sizeof(unsigned) * nslots_));
    d_status_ = static_cast<uint32_t*>(dalloc(sizeof(uint32_t)));
    const int cmax = *std::max_element(F_.begin(), F_.end());
    const size_t ndone = static_cast<size_t>(Bmax_) * ((cmax + 31) / 32);
    d_stat_work_ = static_cast<double*>(dalloc(sizeof(double) * Bmax_ * fxk::kMaxStatSlices * cmax * 2));
    d_stat_done_ = static_cast<unsigned*>(dalloc(sizeof(unsigned) * ndone));
    if (!d_sums_ || !d_amax_ || !d_status_ || !d_stat_work_ || !d_stat_done_)
        return fail(kInternal, "cudaMalloc: control buffers");
    cudaMemset(d_status_, 0, sizeof(uint32_t));
    cudaMemset(d_stat_done_, 0, sizeof(unsigned) * ndone);
    std::vector<float> g = gaussian1d(tz_), gy = gaussian1d(ty_), gx = gaussian1d(tx_);
    g.insert(g.end(), gy.begin(), gy.end());
    g.insert(g.end(), gx.begin(), gx.end());
    Status st = upload(d_gauss_, g, this, allocs_);
    if (!st.ok()) return st;
    if ((st = upload(d_head_w_, head_w_, this, allocs_)).code) return st;
    if ((st = upload(d_head_b_, head_b_, this, allocs_)).code) return st;
    return cuda_status(cudaDeviceSynchronize(), "allocation");
}

Status Net::create(const std::string& path, const int tile[3], int max_batch, int precision, int device) {
    tz_ = tile[0];
    ty_ = tile[1];
    tx_ = tile[2];
    Bmax_ = max_batch;
    prec_ = precision;
    dev_ = device;
    if (tz_ <= 0 || ty_ <= 0 || tx_ <= 0 || max_batch <= 0) return fail(kInvalid, "net: tile and max_batch must be positive");
    if (precision < 0 || precision > 2) return fail(kInvalid, "net: precision must be bf16 (0), fp8 (1) or f16 (2)");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return fail(kInvalid, "net: CUDA device " + std::to_string(device) + " not available");
    Status st = cuda_status(cudaSetDevice(device), "cudaSetDevice");
    if (!st.ok()) return st;
    cudaDeviceProp prop{};
    cudaGetDeviceProperties(&prop, device);
    if (prop.major != 10) return fail(kUnsupported, "net: needs an sm_100 (B200-class) GPU, found sm_" +
                                                        std::to_string(prop.major) + std::to_string(prop.minor));
    sm_count_ = prop.multiProcessorCount;
    WeightMap wm;
    std::string err = load_fxweights(path, wm);
    if (!err.empty()) return fail(err.find("open") != std::string::npos ? kIo : kDecode, err);
    if ((st = parse(wm)).code) return st;
    {
        int k = 0;
        for (auto* v : {&enc_, &up_, &dec_})
            for (Layer& L : *v) L.idx = k++;
    }
    // the grid of every level: each stage halves the axes of its mask, which must divide evenly
    lv_.assign(S_, ActGeom{});
    lv_[0] = {tz_, ty_, tx_};
    for (int lvl = 1; lvl < S_; ++lvl) {
        const ActGeom& a = lv_[lvl - 1];
        const int m = smask_[lvl];
        if (((m & 4) && a.D % 2) || ((m & 2) && a.H % 2) || ((m & 1) && a.W % 2))
            return fail(kInvalid, "tile (" + std::to_string(tz_) + ", " + std::to_string(ty_) + ", " + std::to_string(tx_) +
                                      ") does not halve evenly through the net's " + std::to_string(S_) + " stages");
        lv_[lvl] = {(m & 4) ? a.D / 2 : a.D, (m & 2) ? a.H / 2 : a.H, (m & 1) ? a.W / 2 : a.W};
    }
    for (int s = 0; s < S_; ++s)
        if (F_[s] % 16) return fail(kUnsupported, "net: stage features must be multiples of 16");
    if (F_[0] > 64) return fail(kUnsupported, "net: first stage wider than 64 channels");
    if ((st = cuda_status(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate")).code) return st;
    if ((st = alloc()).code) return st;
    for (auto* v : {&enc_, &up_, &dec_})
        for (Layer& L : *v)
            if ((st = build_layer(L, t16())).code) return st;
    amax_.assign(nslots_, 0.f);
    return ok();
}

// ---- one conv launch ----------------------------------------------------------------------
Status Net::run_conv(Layer& L, int q, const uint8_t* in_ptr, int64_t in_bs, int64_t in_gs, uint8_t* out_ptr,
                     int64_t out_bs, int64_t out_gs, int out_type, float out_qscale, unsigned* amax, int nb,
                     cudaStream_t s) {
    ProfEv ev{};
    if (profile_) {
        const ActGeom gi = level(L.lin), go = level(L.lout);
        const double vin = static_cast<double>(gi.D) * gi.H * gi.W, vout = static_cast<double>(go.D) * go.H * go.W;
        // algorithmic FLOPs = 2 x MACs: conv 27 Cin Cout Vout, transposed conv Cin Cout Vout
        // (a strided projection counts its AvgPool as 8 taps of the conv it runs as)
        const double taps = L.kind == Layer::kProj ? (L.stride == 2 ? 8.0 : 1.0) : 27.0;
        const double nph = static_cast<double>(1 << __builtin_popcount(static_cast<unsigned>(L.smask)));
        ev.flops = L.kind == Layer::kUp ? 2.0 * L.Cin * L.Cout * nph * vin * nb : 2.0 * taps * L.Cin * L.Cout * vout * nb;
        ev.optype = q;
        ev.layer = L.idx;
        cudaEventCreate(&ev.a);
        cudaEventCreate(&ev.b);
        cudaEventRecord(ev.a, s);
    }
    Status st = launch_layer(L, q, level(L.lin), level(L.lout), in_ptr, in_bs, in_gs, out_ptr, out_bs, out_gs, out_type,
                             out_qscale, amax, nb, sm_count_, d_status_, s);
    if (profile_) {
        cudaEventRecord(ev.b, s);
        prof_.push_back(ev);
    }
    return st;
}

void Net::profile(bool on) { profile_ = on; }

Status Net::profile_read(ProfileTotals& out, double* per, int cap, std::vector<double>* per_layer) {
    out = ProfileTotals{};
    if (per_layer) per_layer->assign(enc_.size() + up_.size() + dec_.size(), 0.0);
    int k = 0;
    for (ProfEv& e : prof_) {
        cudaError_t err = cudaEventSynchronize(e.b);
        if (err != cudaSuccess) return cuda_status(err, "profile");
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e.a, e.b);
        out.conv_ms += ms;
        out.conv_flops += e.flops;
        if (e.optype == fxk::kOpE4M3) out.fp8_flops += e.flops;
        ++out.conv_launches;
        if (per && k < cap) {
            per[2 * k] = ms;
            per[2 * k + 1] = e.flops;
        }
        if (per_layer && e.layer >= 0 && e.layer < static_cast<int>(per_layer->size())) (*per_layer)[e.layer] += ms;
        ++k;
        cudaEventDestroy(e.a);
        cudaEventDestroy(e.b);
    }
    prof_.clear();
    return ok();
}

Status launch_layer(Layer& L, int q, ActGeom gin, ActGeom gout, const uint8_t* in_ptr, int64_t in_bs, int64_t in_gs,
                    uint8_t* out_ptr, int64_t out_bs, int64_t out_gs, int out_type, float out_qscale, unsigned* amax,
                    int nb, int sm_count_, uint32_t* d_status_, cudaStream_t s, bool per_column, uint64_t wait_ns,
                    int stall_first_wait) {
    DevProgram& dp = L.prog[q];
    if (!dp.built) return fail(kInternal, L.name + ": program not built");
    static thread_local fxk::ConvParams p;  // ~22 KB: kept off the stack
    p = fxk::ConvParams{};
    const ActGeom& rs = dp.rowspace;
    if ((L.kind == Layer::kConv || L.kind == Layer::kProj) && L.stride == 2) {
        const int64_t ps = gout.gs();
        const int nph = 1 << __builtin_popcount(static_cast<unsigned>(L.smask));
        for (int phi = 0; phi < nph; ++phi) p.src[phi] = {in_ptr + phi * ps, in_bs, in_gs, gout.rows()};
    } else {
        p.src[0] = {in_ptr, in_bs, in_gs, gin.rows()};
    }
    std::copy(dp.host.stages.begin(), dp.host.stages.end(), p.stages);
    std::copy(dp.host.mmas.begin(), dp.host.mmas.end(), p.mmas);
    p.wpack = dp.wpack;
    p.wtile_bytes = dp.host.wtile_bytes;
    p.n_stages = static_cast<int32_t>(dp.host.stages.size());
    p.n_mmas = static_cast<int32_t>(dp.host.mmas.size());
    p.optype = dp.optype;
    p.batch = nb;
    p.Dp = rs.D + 2;
    p.Hp = rs.H + 2;
    p.Wp = rs.W + 2;
    const int64_t P2 = static_cast<int64_t>(p.Hp) * p.Wp;
    p.row_begin = P2;
    p.row_end = static_cast<int64_t>(p.Dp - 1) * P2;
    p.R = dp.R;
    p.block_rows = dp.block_rows;
    p.fold = dp.fold ? 1 : 0;
    p.zfold = dp.zfold ? 1 : 0;
    if (dp.zfold) {
        p.zseg = dp.zseg;
        p.zplanes = dp.zplanes;
        p.zkstride = dp.host.zkstride;
        p.bres_bytes = dp.host.bres_bytes;
        p.bres_off = static_cast<int32_t>((static_cast<size_t>(dp.host.n_pipe) * dp.host.stage_bytes +
                                           fxk::conv_tc_ctl_bytes() + 127) / 128 * 128);
    }
    p.n_units_m = dp.n_units_m;
    p.n_tiles = dp.host.n_tiles;
    p.N_tile = dp.N_tile;
    p.acc_slots = dp.acc_slots;
    p.tmem_cols = dp.tmem_cols;
    p.n_pipe = dp.host.n_pipe;
    p.stage_bytes = dp.host.stage_bytes;
    p.stage_a_bytes = dp.host.stage_a_bytes;
    p.col_scale = dp.colscale;
    p.out = out_ptr;
    p.out_batch_stride = out_bs;
    p.out_group_stride = out_gs;
    p.status = d_status_;
    p.wait_ns = wait_ns;
    p.stall_first_wait = stall_first_wait;
    p.trace = g_conv_trace;
    if (L.kind == Layer::kUp) {
        p.mode = fxk::kModeUpsample;
        p.up_mask = L.smask;
        p.bias = dp.bias;
        p.out_type = out_type;
        p.out_qscale = out_qscale;
        p.cout = L.Cout;
        p.oHp = gout.H + 2;
        p.oWp = gout.W + 2;
        p.amax = amax;
    } else {
        p.mode = fxk::kModePrenorm;
        p.stats = L.d_partials;
        p.stats_C = L.Cout;
        p.acc_scale = dp.acc_scale;  // used when there is no per-column table
        if (!per_column) {
            p.col_scale = nullptr;
            L.cur_ratio = dp.ratio;
        } else {
            L.cur_ratio = nullptr;
        }
        p.stat_recs = (!dp.fold && dp.N_tile >= 32 && (dp.R == 1 || dp.N_tile <= 64)) ? fxk::kStatRecsPerUnit / 2
                                                                                        : fxk::kStatRecsPerUnit;
    }
    const int64_t units = static_cast<int64_t>(nb) * p.n_units_m * p.n_tiles;
    const int grid = static_cast<int>(std::min<int64_t>(units, sm_count_));
    if (p.mode == fxk::kModePrenorm) {
        // x fold: records per unit, each rewritten by every launch; otherwise records per CTA that the
        // epilogue adds into (zero before the launch: cleared by the statistics pass that reads them,
        // or here when the previous launch was not followed by one)
        L.nrec = (dp.fold ? dp.n_units_m : grid) * p.stat_recs;
        if (L.nrec > L.nrec_cap) return fail(kInternal, L.name + ": statistics buffer too small");
        if (L.partials_dirty)
            cudaMemsetAsync(L.d_partials, 0, sizeof(float) * static_cast<size_t>(nb) * L.nrec_cap * L.Cout * 2, s);
        L.partials_dirty = true;
    }
    return cuda_status(fxk::launch_conv_tc(p, grid, dp.smem(), s), L.name.c_str());
}

Status Net::finalize_in(Layer& L, int nb, cudaStream_t s) {
    const ActGeom g = level(L.lout);
    const double count = static_cast<double>(g.D) * g.H * g.W;
    L.partials_dirty = false;  // the statistics pass leaves the records it reads at zero
    return cuda_status(fxk::launch_in_finalize(L.d_partials, nb, L.nrec, L.Cout, count, L.d_gamma, L.d_beta,
                                               L.cur_ratio, kEps, d_stat_work_, d_stat_done_, L.d_ss, s),
                       "in_finalize");
}

// ---- forward -----------------------------------------------------------------------------------
// Operand precision of one layer: e4m3 for fp8 nets once calibrated, except the first conv
// (always bf16) and layers whose input channels do not fill whole e4m3 MMA K-steps (32).
int Net::layer_q(const Layer& L, bool calib) const {
    if (prec_ != 1 || calib || L.kind == Layer::kFirst || L.keep16) return t16();
    return L.Cin % 32 == 0 ? fxk::kOpE4M3 : t16();
}

Status Net::forward(const uint8_t* vol, int64_t dz, int64_t dy, int64_t dx, const fxk::TileOrigin* d_tiles, int nb,
                    int channel, int sigmoid, float* acc, float* prob, bool calib, cudaStream_t s,
                    int64_t acc_z_shift, int64_t acc_dz, const uint8_t* d_tta, float tta_scale) {
    if (nb < 1 || nb > Bmax_) return fail(kInvalid, "forward: batch out of range");
    if (prec_ == 1 && !calib && !calibrated_) return fail(kInvalid, "forward: fp8 net used before fx_net_calibrate");
    Status st;
    const ActGeom g0 = level(0);
    if ((st = cuda_status(cudaMemsetAsync(d_sums_, 0, sizeof(unsigned long long) * 2 * nb, s), "memset")).code) return st;
    if (norm_ == 1 && (st = cuda_status(cudaMemsetAsync(d_hist_, 0, sizeof(unsigned) * 256 * nb, s), "memset")).code)
        return st;
    if ((st = cuda_status(fxk::launch_tile_sums(vol, dz, dy, dx, d_tiles, nb, tile(), d_sums_, s, norm_ == 1 ? d_hist_ : nullptr),
                          "tile_sums"))
            .code)
        return st;
    const int64_t pvox = tile().count();
    if ((st = cuda_status(fxk::launch_tile_lut(d_sums_, d_hist_, nb, pvox, norm_, d_luts_, nullptr, s), "tile_lut")).code)
        return st;
    if ((st = cuda_status(fxk::launch_tile_norm(vol, dz, dy, dx, d_tiles, nb, tile(), d_sums_, l0_, 2 * g0.gs(), g0.gs(), t16(), nullptr,
                                                s, d_tta, d_luts_),
                          "tile_norm"))
            .code)
        return st;
    auto amax_slot = [&](int k) -> unsigned* { return calib ? d_amax_ + k : nullptr; };
    auto qof = [&](const Layer& L) { return layer_q(L, calib); };
    // bytes per batch item of a tensor of C channels at level lvl stored with precision q
    auto cgof = [](int q) { return q == fxk::kOpE4M3 ? 16 : 8; };
    auto bstride = [&](int lvl, int C, int q) { return static_cast<int64_t>(C / cgof(q)) * level(lvl).gs(); };
    // destination written for consumer layer `cons` (its precision and input scale)
    auto dest = [&](uint8_t* ptr, int lvl, int Cbuf, int ch0, const Layer& cons) {
        const int q = qof(cons);
        fxk::NormDest d{};
        d.ptr = ptr + static_cast<int64_t>(ch0 / cgof(q)) * level(lvl).gs();
        d.batch_stride = bstride(lvl, Cbuf, q);
        d.group_stride = level(lvl).gs();
        d.dtype = q;
        d.qscale = q == fxk::kOpE4M3 ? 1.f / cons.in_scale : 1.f;
        return d;
    };
    auto phase_dest = [&](int lvl, const Layer& cons) {
        const int q = qof(cons);
        fxk::NormDest d{};
        const ActGeom gn = level(lvl + 1);
        d.ptr = ph_[lvl];
        d.phase = smask_[lvl + 1];
        d.pHp = gn.H + 2;
        d.pWp = gn.W + 2;
        d.phase_stride = gn.gs();
        d.group_stride = (1 << __builtin_popcount(static_cast<unsigned>(smask_[lvl + 1]))) * gn.gs();
        d.batch_stride = static_cast<int64_t>(F_[lvl] / cgof(q)) * d.group_stride;
        d.dtype = q;
        d.qscale = q == fxk::kOpE4M3 ? 1.f / cons.in_scale : 1.f;
        return d;
    };
    auto norm = [&](Layer& L, fxk::NormDest d0, fxk::NormDest d1, int slot) -> Status {
        Status r = finalize_in(L, nb, s);
        if (!r.ok()) return r;
        const ActGeom g = level(L.lout);
        return cuda_status(fxk::launch_norm_act(pn_[L.lout], static_cast<int64_t>(L.Cout / 8) * g.gs(), g.gs(),
                                                {g.D, g.H, g.W}, L.Cout, nb, L.d_ss, kSlope, d0, d1, amax_slot(slot), s),
                           "norm_act");
    };
    const fxk::NormDest none{};
    // encoder: residual stages (stem + BasicBlockD)
    if (resenc_) {
        const Layer& stem = enc_[0];
        const ActGeom g0l = level(0);
        const int64_t pn0 = static_cast<int64_t>(F_[0] / 8) * g0l.gs();
        // f16 copy of a level's block input (identity / pooled residual source)
        auto f16dest = [&](uint8_t* ptr, int lvl, int C) {
            fxk::NormDest d{};
            d.ptr = ptr;
            d.batch_stride = static_cast<int64_t>(C / 8) * level(lvl).gs();
            d.group_stride = level(lvl).gs();
            d.dtype = fxk::kOpF16;
            d.qscale = 1.f;
            return d;
        };
        if ((st = run_conv(enc_[0], qof(stem), l0_, 2 * g0.gs(), g0.gs(), pn_[0], pn0, g0l.gs(), 0, 1.f, nullptr, nb, s)).code)
            return st;
        if ((st = norm(enc_[0], dest(act_[0], 0, F_[0], 0, enc_[blocks_[0].c1]), f16dest(xf_[0], 0, F_[0]),
                       blocks_[0].slot_x))
                .code)
            return st;
        for (size_t k = 0; k < blocks_.size(); ++k) {
            const ResBlock& K = blocks_[k];
            const int lv = K.stage;
            const ActGeom g = level(lv);
            const int64_t pbs = static_cast<int64_t>(F_[lv] / 8) * g.gs();
            Layer& L1 = enc_[K.c1];
            Layer& L2 = enc_[K.c2];
            const int q1 = qof(L1), q2 = qof(L2);
            // conv1 (and the projection) read the block input: the phase-split copy when strided
            const uint8_t* in1;
            int64_t ibs, igs;
            if (K.stride == 2) {
                in1 = ph_[lv - 1];
                igs = (1 << __builtin_popcount(static_cast<unsigned>(smask_[lv]))) * g.gs();
                ibs = static_cast<int64_t>(L1.Cin / cgof(q1)) * igs;
            } else {
                in1 = act_[lv];
                igs = g.gs();
                ibs = bstride(lv, L1.Cin, q1);
            }
            if ((st = run_conv(L1, q1, in1, ibs, igs, pn_[lv], pbs, g.gs(), 0, 1.f, nullptr, nb, s)).code) return st;
            if ((st = norm(L1, dest(h_[lv], lv, F_[lv], 0, L2), none, K.slot_h)).code) return st;
            if ((st = run_conv(L2, q2, h_[lv], bstride(lv, F_[lv], q2), g.gs(), pn_[lv], pbs, g.gs(), 0, 1.f, nullptr,
                               nb, s))
                    .code)
                return st;
            if ((st = finalize_in(L2, nb, s)).code) return st;
            fxk::BlockOut bo{};
            if (K.proj >= 0) {
                Layer& Lp = enc_[K.proj];
                const int qp = qof(Lp);
                const int64_t pibs = K.stride == 2 ? static_cast<int64_t>(Lp.Cin / cgof(qp)) * igs : bstride(lv, Lp.Cin, qp);
                if ((st = run_conv(Lp, qp, in1, pibs, igs, pnx_[lv], pbs, g.gs(), 0, 1.f, nullptr, nb, s)).code) return st;
                if ((st = finalize_in(Lp, nb, s)).code) return st;
                bo.res = pnx_[lv];
                bo.res_ss = Lp.d_ss;
            } else if (K.avgpool) {
                const ActGeom gi = level(lv - 1);
                if ((st = cuda_status(fxk::launch_avgpool2_f16(xf_[lv - 1], static_cast<int64_t>(F_[lv - 1] / 8) * gi.gs(),
                                                               gi.gs(), {gi.D, gi.H, gi.W}, res_[lv], pbs, g.gs(),
                                                               F_[lv] / 8, nb, s),
                                      "avgpool"))
                        .code)
                    return st;
                bo.res = res_[lv];
            } else {
                bo.res = xf_[lv];
            }
            bo.res_bs = pbs;
            bo.res_gs = g.gs();
            if (K.se) {
                if ((st = cuda_status(fxk::launch_sse_gate(pn_[lv], pbs, g.gs(), L2.d_ss, K.d_sse_w, K.sse_b,
                                                           {g.D, g.H, g.W}, F_[lv], nb, sg_[lv], s),
                                      "sse_gate"))
                        .code)
                    return st;
                bo.cgate = K.d_cgate;
                bo.sgate = sg_[lv];
            }
            bo.pre = pn_[lv];
            bo.pre_bs = pbs;
            bo.pre_gs = g.gs();
            bo.ss = L2.d_ss;
            bo.slope = kSlope;
            bo.g = {g.D, g.H, g.W};
            bo.C = F_[lv];
            bo.B = nb;
            const bool last_in_stage = k + 1 == blocks_.size() || blocks_[k + 1].stage != lv;
            int slot;
            if (!last_in_stage) {  // next block of the stage: its conv1 operands + the f16 residual copy
                bo.d[0] = dest(act_[lv], lv, F_[lv], 0, enc_[blocks_[k + 1].c1]);
                bo.d[1] = f16dest(xf_[lv], lv, F_[lv]);
                slot = blocks_[k + 1].slot_x;
            } else if (lv < S_ - 1) {  // next stage (phase-split), decoder skip half, f16 copy
                const ResBlock& Kn = blocks_[k + 1];
                bo.d[0] = phase_dest(lv, enc_[Kn.c1]);
                bo.d[1] = dest(cat_[lv], lv, 2 * F_[lv], F_[lv], dec_[lv * nconv_]);
                if (Kn.avgpool) bo.d[2] = f16dest(xf_[lv], lv, F_[lv]);
                slot = Kn.slot_x;
            } else {  // the bottleneck: input of the first transposed conv
                bo.d[0] = dest(act_[lv], lv, F_[lv], 0, up_[S_ - 2]);
                slot = nslots_ - 1;
            }
            bo.amax = amax_slot(slot);
            if ((st = cuda_status(fxk::launch_block_out(bo, s), "block_out")).code) return st;
        }
    } else {
        // encoder
        for (int lv = 0; lv < S_; ++lv) {
            const ActGeom g = level(lv);
            const int64_t pn_bs = static_cast<int64_t>(F_[lv] / 8) * g.gs();
            for (int i = 0; i < nconv_; ++i) {
                Layer& L = enc_[lv * nconv_ + i];
                const int q = qof(L);
                const uint8_t* in;
                int64_t ibs, igs;
                if (L.kind == Layer::kFirst) {
                    in = l0_;
                    ibs = 2 * g0.gs();
                    igs = g0.gs();
                } else if (i == 0) {  // stride 2: phase-split copy of the previous stage's output
                    in = ph_[lv - 1];
                    igs = (1 << __builtin_popcount(static_cast<unsigned>(smask_[lv]))) * g.gs();
                    ibs = static_cast<int64_t>(F_[lv - 1] / cgof(q)) * igs;
                } else {
                    in = act_[lv];
                    ibs = bstride(lv, F_[lv], q);
                    igs = g.gs();
                }
                if ((st = run_conv(L, q, in, ibs, igs, pn_[lv], pn_bs, g.gs(), 0, 1.f, nullptr, nb, s)).code) return st;
                if (i < nconv_ - 1) {
                    if ((st = norm(L, dest(act_[lv], lv, F_[lv], 0, enc_[lv * nconv_ + i + 1]), none, lv)).code) return st;
                } else if (lv < S_ - 1) {
                    const Layer& dcat = dec_[lv * nconv_];
                    if ((st = norm(L, dest(cat_[lv], lv, 2 * F_[lv], F_[lv], dcat), phase_dest(lv, enc_[(lv + 1) * nconv_]),
                                   S_ + lv))
                            .code)
                        return st;
                } else {
                    if ((st = norm(L, dest(act_[lv], lv, F_[lv], 0, up_[S_ - 2]), none, S_ + lv)).code) return st;
                }
            }
        }
    }
    // decoder
    for (int lv = S_ - 2; lv >= 0; --lv) {
        const ActGeom g = level(lv);
        Layer& U = up_[lv];
        const Layer& dcat = dec_[lv * nconv_];
        const int qu = qof(U), qc = qof(dcat);
        if ((st = run_conv(U, qu, act_[lv + 1], bstride(lv + 1, F_[lv + 1], qu), level(lv + 1).gs(), cat_[lv],
                           bstride(lv, 2 * F_[lv], qc), g.gs(), qc, qc == fxk::kOpE4M3 ? 1.f / dcat.in_scale : 1.f,
                           amax_slot(2 * S_ + lv), nb, s))
                .code)
            return st;
        const int64_t pn_bs = static_cast<int64_t>(F_[lv] / 8) * g.gs();
        for (int i = 0; i < nconv_; ++i) {
            Layer& L = dec_[lv * nconv_ + i];
            const int q = qof(L);
            const uint8_t* in = i == 0 ? cat_[lv] : act_[lv];
            const int64_t ibs = i == 0 ? bstride(lv, 2 * F_[lv], q) : bstride(lv, F_[lv], q);
            if ((st = run_conv(L, q, in, ibs, g.gs(), pn_[lv], pn_bs, g.gs(), 0, 1.f, nullptr, nb, s)).code) return st;
            if (i < nconv_ - 1) {
                if ((st = norm(L, dest(act_[lv], lv, F_[lv], 0, dec_[lv * nconv_ + i + 1]), none, 3 * S_ + lv)).code)
                    return st;
            } else if (lv > 0) {
                if ((st = norm(L, dest(act_[lv], lv, F_[lv], 0, up_[lv - 1]), none, 4 * S_ + lv)).code) return st;
            } else {
                if ((st = finalize_in(L, nb, s)).code) return st;
                fxk::HeadParams h{};
                h.pre = pn_[0];
                h.pre_batch_stride = pn_bs;
                h.pre_group_stride = g.gs();
                h.Pz = tz_;
                h.Py = ty_;
                h.Px = tx_;
                h.C = F_[0];
                h.B = nb;
                h.ncls = ncls_;
                h.channel = channel;
                h.sigmoid = sigmoid;
                h.ss = L.d_ss;
                h.slope = kSlope;
                h.wh = d_head_w_;
                h.bh = d_head_b_;
                h.gz = d_gauss_;
                h.gy = d_gauss_ + tz_;
                h.gx = d_gauss_ + tz_ + ty_;
                h.tiles = d_tiles;
                h.tta = d_tta;
                h.tta_scale = tta_scale;
                h.acc = acc;
                h.dz = dz;
                h.dy = dy;
                h.dx = dx;
                h.acc_z_shift = acc_z_shift;
                h.acc_dz = acc_dz < 0 ? dz : acc_dz;
                h.acc_y_shift = acc_y_shift_;
                h.acc_dy = acc_dy_;
                h.acc_x_shift = acc_x_shift_;
                h.acc_dx = acc_dx_;
                h.prob = prob;
                if ((st = cuda_status(fxk::launch_head_blend(h, s), "head_blend")).code) return st;
            }
        }
    }
    return ok();
}

// ---- calibration ------------------------------------------------------------------------------
Status Net::set_scales_from_amax() {
    auto sc = [&](int k) { return std::max(amax_[k], 1e-8f) / kE4M3Max; };
    if (resenc_) {
        // block b's input (conv1, projection) and conv2 input; a stage's last block output is the
        // next stage's first block input and the decoder's skip half at that level
        int first_of_stage[64] = {};
        for (int k = static_cast<int>(blocks_.size()) - 1; k >= 0; --k) first_of_stage[blocks_[k].stage] = k;
        for (const ResBlock& K : blocks_) {
            enc_[K.c1].in_scale = sc(K.slot_x);
            enc_[K.c2].in_scale = sc(K.slot_h);
            if (K.proj >= 0) enc_[K.proj].in_scale = sc(K.slot_x);
        }
        const int last = nslots_ - 1;  // the last stage's output
        for (int lvl = 0; lvl < S_ - 1; ++lvl) {
            const int skip = blocks_[first_of_stage[lvl + 1]].slot_x;
            dec_[lvl * nconv_].in_scale = std::max(sc(skip), sc(2 * S_ + lvl));
            for (int i = 1; i < nconv_; ++i) dec_[lvl * nconv_ + i].in_scale = sc(3 * S_ + lvl);
            up_[lvl].in_scale = lvl == S_ - 2 ? sc(last) : sc(4 * S_ + lvl + 1);
        }
        return ok();
    }
    for (int s = 0; s < S_; ++s) {
        for (int i = 1; i < nconv_; ++i) enc_[s * nconv_ + i].in_scale = sc(s);  // nA
        if (s + 1 < S_) enc_[(s + 1) * nconv_].in_scale = sc(S_ + s);           // skip -> phase copy
    }
    for (int lvl = 0; lvl < S_ - 1; ++lvl) {
        const float scat = std::max(sc(S_ + lvl), sc(2 * S_ + lvl));
        dec_[lvl * nconv_].in_scale = scat;
        for (int i = 1; i < nconv_; ++i) dec_[lvl * nconv_ + i].in_scale = sc(3 * S_ + lvl);
        up_[lvl].in_scale = lvl == S_ - 2 ? sc(S_ + S_ - 1) : sc(4 * S_ + lvl + 1);
    }
    return ok();
}

Status Net::calibrate(const uint8_t* host_patches, int n) {
    if (prec_ != 1) return fail(kInvalid, "calibrate: net is not fp8");
    if (n < 1) return fail(kInvalid, "calibrate: need at least one patch");
    cudaSetDevice(dev_);
    const size_t pv = static_cast<size_t>(tile().count());
    uint8_t* d_vol = static_cast<uint8_t*>(dalloc(pv * Bmax_));
    if (!d_vol) return fail(kInternal, "cudaMalloc: calibration patches");
    std::vector<fxk::TileOrigin> org(Bmax_);
    for (int b = 0; b < Bmax_; ++b) org[b] = {static_cast<int64_t>(b) * tz_, 0, 0};
    fxk::TileOrigin* d_org = nullptr;
    Status st = upload(d_org, org, this, allocs_);
    if (!st.ok()) return st;
    cudaMemsetAsync(d_amax_, 0, sizeof(unsigned) * nslots_, stream_);
    for (int i0 = 0; i0 < n; i0 += Bmax_) {
        const int nb = std::min(Bmax_, n - i0);
        if ((st = cuda_status(cudaMemcpyAsync(d_vol, host_patches + pv * i0, pv * nb, cudaMemcpyHostToDevice, stream_),
                              "H2D calibration"))
                .code)
            return st;
        if ((st = forward(d_vol, static_cast<int64_t>(nb) * tz_, ty_, tx_, d_org, nb, 1, 0, nullptr, nullptr, true,
                          stream_))
                .code)
            return st;
    }
    std::vector<unsigned> bits(nslots_);
    if ((st = cuda_status(cudaMemcpyAsync(bits.data(), d_amax_, sizeof(unsigned) * bits.size(), cudaMemcpyDeviceToHost,
                                          stream_),
                          "D2H amax"))
            .code)
        return st;
    if ((st = cuda_status(cudaStreamSynchronize(stream_), "calibration forward")).code) return st;
    if ((st = take_device_status()).code) return fail(st.code, "calibration: " + st.msg);
    for (size_t k = 0; k < bits.size(); ++k) {
        float f;
        std::memcpy(&f, &bits[k], 4);
        amax_[k] = std::max(amax_[k], f);  // running max over calls
    }
    set_scales_from_amax();
    for (auto* v : {&enc_, &up_, &dec_})
        for (Layer& L : *v) {
            L.prog[1] = DevProgram{};  // scales changed: every e4m3 program is stale
            if (layer_q(L, false) != fxk::kOpE4M3) continue;
            if ((st = build_layer(L, 1)).code) return st;
        }
    calibrated_ = true;
    return ok();
}

Status Net::set_act_scales(const float* scales, int n) {
    if (prec_ != 1) return fail(kInvalid, "set_act_scales: net is not fp8");
    const int total = static_cast<int>(enc_.size() + up_.size() + dec_.size());
    if (n != total) return fail(kInvalid, "set_act_scales: expected " + std::to_string(total) + " scales");
    for (int i = 0; i < n; ++i)
        if (!(scales[i] > 0.f) || !std::isfinite(scales[i])) return fail(kInvalid, "set_act_scales: scales must be finite and > 0");
    cudaSetDevice(dev_);
    int k = 0;
    Status st;
    for (auto* v : {&enc_, &up_, &dec_})
        for (Layer& L : *v) L.in_scale = scales[k++];
    for (auto* v : {&enc_, &up_, &dec_})
        for (Layer& L : *v) {
            L.prog[1] = DevProgram{};  // scales changed: every e4m3 program is stale
            if (layer_q(L, false) != fxk::kOpE4M3) continue;
            if ((st = build_layer(L, 1)).code) return st;
        }
    calibrated_ = true;
    return ok();
}

Status Net::set_layer_precision(const int* q, int n) {
    const int total = static_cast<int>(enc_.size() + up_.size() + dec_.size());
    if (n != total) return fail(kInvalid, "set_layer_precision: expected " + std::to_string(total) + " entries");
    for (int i = 0; i < n; ++i)
        if (q[i] != fxk::kOpE4M3 && q[i] != t16())
            return fail(kInvalid, "set_layer_precision: entries must be fp8 or the net's 16-bit type");
    if (prec_ != 1) {
        for (int i = 0; i < n; ++i)
            if (q[i] == fxk::kOpE4M3) return fail(kInvalid, "set_layer_precision: the net is not fp8");
        return ok();
    }
    cudaSetDevice(dev_);
    int k = 0;
    for (auto* v : {&enc_, &up_, &dec_})
        for (Layer& L : *v) L.keep16 = q[k++] != fxk::kOpE4M3;
    if (!calibrated_) return ok();  // calibration builds the e4m3 programs
    Status st;
    for (auto* v : {&enc_, &up_, &dec_})
        for (Layer& L : *v)
            if (layer_q(L, false) == fxk::kOpE4M3 && !L.prog[1].built && (st = build_layer(L, 1)).code) return st;
    return ok();
}

Status Net::calibrate_schedule(const uint8_t* host_patches, int n, double min_dice, double max_abs, double* dice_out,
                               double* maxabs_out) {
    if (prec_ != 1) return fail(kInvalid, "calibrate_schedule: net is not fp8");
    if (n < 1 || !host_patches) return fail(kInvalid, "calibrate_schedule: need at least one patch");
    if (!(min_dice >= 0.0 && min_dice <= 1.0)) return fail(kInvalid, "calibrate_schedule: min_dice must be in [0, 1]");
    Status st;
    if (!calibrated_ && (st = calibrate(host_patches, n)).code) return st;
    cudaSetDevice(dev_);
    const size_t pv = static_cast<size_t>(tile().count());
    auto* d_vol = static_cast<uint8_t*>(dalloc(pv * n));
    auto* d_ref = static_cast<float*>(dalloc(sizeof(float) * pv * n));
    auto* d_cur = static_cast<float*>(dalloc(sizeof(float) * pv * n));
    auto* d_cmp = static_cast<unsigned long long*>(dalloc(sizeof(unsigned long long) * 4));
    auto* d_org = static_cast<fxk::TileOrigin*>(dalloc(sizeof(fxk::TileOrigin) * Bmax_));
    if (!d_vol || !d_ref || !d_cur || !d_cmp || !d_org) return fail(kInternal, "cudaMalloc: schedule search buffers");
    std::vector<fxk::TileOrigin> org(Bmax_);
    for (int b = 0; b < Bmax_; ++b) org[b] = {static_cast<int64_t>(b) * tz_, 0, 0};
    cudaMemcpyAsync(d_org, org.data(), sizeof(fxk::TileOrigin) * Bmax_, cudaMemcpyHostToDevice, stream_);
    cudaMemcpyAsync(d_vol, host_patches, pv * n, cudaMemcpyHostToDevice, stream_);
    const int nl = static_cast<int>(enc_.size() + up_.size() + dec_.size());
    std::vector<int> elig;
    for (int k = 0; k < nl; ++k) {
        Layer& L = const_cast<Layer&>(*layer_at(k));
        const bool saved = L.keep16;
        L.keep16 = false;
        if (layer_q(L, false) == fxk::kOpE4M3) elig.push_back(k);
        L.keep16 = saved;
    }
    const int sig = ncls_ == 1 ? 1 : 0;
    // every tile of the calibration set through the net with schedule q8 (1 = e4m3), probabilities into out
    auto run = [&](const std::vector<char>& q8, float* out) -> Status {
        std::vector<int> q(nl, t16());
        for (int k = 0; k < nl; ++k)
            if (q8[k]) q[k] = fxk::kOpE4M3;
        Status r = set_layer_precision(q.data(), nl);
        if (!r.ok()) return r;
        for (int i0 = 0; i0 < n; i0 += Bmax_) {
            const int nb = std::min(Bmax_, n - i0);
            if ((r = forward(d_vol + pv * i0, static_cast<int64_t>(nb) * tz_, ty_, tx_, d_org, nb, 1, sig, nullptr,
                             out + pv * i0, false, stream_))
                    .code)
                return r;
        }
        return take_device_status();
    };
    // Dice of the 0.5-thresholded masks and max |dp| of d_cur against d_ref
    auto compare = [&](double& dice, double& mx) -> Status {
        cudaMemsetAsync(d_cmp, 0, sizeof(unsigned long long) * 4, stream_);
        Status r = cuda_status(fxk::launch_prob_compare(d_ref, d_cur, static_cast<int64_t>(pv) * n, d_cmp,
                                                        reinterpret_cast<unsigned*>(d_cmp + 3), stream_),
                               "prob_compare");
        if (!r.ok()) return r;
        unsigned long long h[4] = {0, 0, 0, 0};
        if ((r = cuda_status(cudaMemcpyAsync(h, d_cmp, sizeof h, cudaMemcpyDeviceToHost, stream_), "D2H")).code) return r;
        if ((r = cuda_status(cudaStreamSynchronize(stream_), "compare")).code) return r;
        dice = h[0] + h[1] == 0 ? 1.0 : 2.0 * static_cast<double>(h[2]) / static_cast<double>(h[0] + h[1]);
        float f;
        const unsigned bits = static_cast<unsigned>(h[3]);
        std::memcpy(&f, &bits, 4);
        mx = f;
        return ok();
    };
    std::vector<char> none(nl, 0), all(nl, 0);
    for (int k : elig) all[k] = 1;
    // conv time per layer on each operand type (one profiled pass each), and the 16-bit yardstick
    const bool was_profiling = profile_;
    std::vector<double> t16, t8;
    profile_ = true;
    st = run(all, d_cur);
    if (st.ok()) {
        ProfileTotals tot;
        st = profile_read(tot, nullptr, 0, &t8);
    }
    if (st.ok()) st = run(none, d_ref);
    if (st.ok()) {
        ProfileTotals tot;
        st = profile_read(tot, nullptr, 0, &t16);
    }
    profile_ = was_profiling;
    if (!st.ok()) return st;
    struct Cand {
        int k;
        double loss2, mx, gain;
    };
    std::vector<Cand> cands;
    for (int k : elig) {
        std::vector<char> q(nl, 0);
        q[k] = 1;
        double d = 1.0, mx = 0.0;
        if ((st = run(q, d_cur)).code || (st = compare(d, mx)).code) return st;
        const double loss = std::max(1.0 - d, 1e-7);
        cands.push_back({k, loss * loss, mx, t16[k] - t8[k]});
    }
    std::sort(cands.begin(), cands.end(), [](const Cand& a, const Cand& b) { return a.gain / a.loss2 > b.gain / b.loss2; });
    const double budget = (1.0 - min_dice) * (1.0 - min_dice);
    std::vector<char> cur(nl, 0);
    std::vector<int> taken;
    double used = 0.0;
    for (const Cand& c : cands) {
        if (c.gain <= 0.0 || (max_abs > 0.0 && c.mx > max_abs) || used + c.loss2 > budget) continue;
        cur[c.k] = 1;
        used += c.loss2;
        taken.push_back(c.k);
    }
    double dice = 1.0, mx = 0.0;
    for (;;) {
        if ((st = run(cur, d_cur)).code || (st = compare(dice, mx)).code) return st;
        if ((dice >= min_dice && (max_abs <= 0.0 || mx <= max_abs)) || taken.empty()) break;
        cur[taken.back()] = 0;
        taken.pop_back();
    }
    if (dice_out) *dice_out = dice;
    if (maxabs_out) *maxabs_out = mx;
    return ok();
}

std::vector<int> Net::layer_precision() const {
    std::vector<int> out;
    for (auto* v : {&enc_, &up_, &dec_})
        for (const Layer& L : *v) out.push_back(layer_q(L, false));
    return out;
}

Status Net::take_device_status() {
    cudaSetDevice(dev_);
    Status st = cuda_status(cudaStreamSynchronize(stream_), "stream");
    if (!st.ok()) return st;
    uint32_t v = 0;
    if ((st = cuda_status(cudaMemcpy(&v, d_status_, 4, cudaMemcpyDeviceToHost), "D2H status")).code) return st;
    if (!v) return ok();
    cudaMemset(d_status_, 0, 4);
    char buf[96];
    std::snprintf(buf, sizeof buf, "device status 0x%x: a kernel's bounded wait timed out", v);
    return fail(kInternal, buf);
}

const Layer* Net::layer_at(int i) const {
    for (auto* v : {&enc_, &up_, &dec_}) {
        if (i >= 0 && i < static_cast<int>(v->size())) return &(*v)[i];
        i -= static_cast<int>(v->size());
    }
    return nullptr;
}

std::vector<double> Net::layer_flops() const {
    std::vector<double> out;
    for (auto* v : {&enc_, &up_, &dec_})
        for (const Layer& L : *v) {
            const ActGeom gi = level(L.lin), go = level(L.lout);
            const double vin = static_cast<double>(gi.D) * gi.H * gi.W, vout = static_cast<double>(go.D) * go.H * go.W;
            const double taps = L.kind == Layer::kProj ? (L.stride == 2 ? 8.0 : 1.0) : 27.0;
            const double nph = static_cast<double>(1 << __builtin_popcount(static_cast<unsigned>(L.smask)));
            out.push_back(L.kind == Layer::kUp ? 2.0 * L.Cin * L.Cout * nph * vin : 2.0 * taps * L.Cin * L.Cout * vout);
        }
    return out;
}

std::vector<float> Net::act_scales() const {
    std::vector<float> out;
    for (auto* v : {&enc_, &up_, &dec_})
        for (const Layer& L : *v) out.push_back(L.in_scale);
    return out;
}

// ---- sliding window ---------------------------------------------------------------------------
Status Net::workspace(size_t vol_bytes, size_t acc_bytes, size_t out_bytes, uint8_t** vol, float** acc,
                      uint8_t** out) {
    auto grow = [&](void** p, size_t& cap, size_t need) -> bool {
        if (need <= cap) return true;
        if (*p) {
            cudaStreamSynchronize(stream_);
            cudaFree(*p);
            allocs_.erase(std::remove(allocs_.begin(), allocs_.end(), *p), allocs_.end());
            *p = nullptr;
            cap = 0;
        }
        void* q = dalloc(need);
        if (!q) return false;
        *p = q;
        cap = need;
        return true;
    };
    if (!grow(reinterpret_cast<void**>(&ws_vol_), ws_vol_cap_, vol_bytes) ||
        !grow(reinterpret_cast<void**>(&ws_acc_), ws_acc_cap_, acc_bytes) ||
        (out_bytes && !grow(reinterpret_cast<void**>(&ws_out_), ws_out_cap_, out_bytes)))
        return fail(kInternal, "cudaMalloc: volume workspace");
    *vol = ws_vol_;
    *acc = ws_acc_;
    if (out) *out = ws_out_;
    return ok();
}

float* Net::profile_buffer(size_t n) {
    if (n <= ws_prof_cap_) return ws_prof_;
    if (ws_prof_) {
        cudaDeviceSynchronize();
        cudaFree(ws_prof_);
        allocs_.erase(std::remove(allocs_.begin(), allocs_.end(), static_cast<void*>(ws_prof_)), allocs_.end());
        ws_prof_ = nullptr;
        ws_prof_cap_ = 0;
    }
    ws_prof_ = static_cast<float*>(dalloc(sizeof(float) * n));
    if (ws_prof_) ws_prof_cap_ = n;
    return ws_prof_;
}

Status Net::predict_tiles(const uint8_t* d_vol, int64_t dz, int64_t dy, int64_t dx, int64_t z_origin, int64_t full_dz,
                          fxk::TileDims tl, double overlap, int channel, int sigmoid, int batch, int64_t tile_begin,
                          int64_t tile_end, float* d_acc, cudaStream_t s, int64_t acc_z_origin, int64_t acc_dz,
                          int tta, const RunOpts& ro) {
    if (tl.z != tz_ || tl.y != ty_ || tl.x != tx_) return fail(kInvalid, "predict: tile differs from the net's tile");
    if (tta > 1 && !patch()) return fail(kUnsupported, "predict: TTA members permute axes and need a cubic tile");
    if (ro.norm < 0 || ro.norm > 2) return fail(kInvalid, "predict: norm must be zscore, pct_minmax or unit255");
    if (batch < 1) batch = 1;
    batch = std::min(batch, Bmax_);
    if (full_dz <= 0) full_dz = dz;
    const int ns = std::max(ro.stacks, 1);
    std::vector<int64_t> zs;
    if (ns == 1) {
        zs = tile_starts(full_dz, tz_, overlap);
    } else {
        // independent stacks along z: each stack's own starts, offset to the stack
        if (full_dz % ns || z_origin != 0 || dz != full_dz)
            return fail(kInvalid, "predict: stacks must divide the whole volume's depth (no z-slabs)");
        const int64_t sd = full_dz / ns;
        if (sd < tz_) return fail(kInvalid, "predict: a stack is thinner than the tile");
        const auto z1 = tile_starts(sd, tz_, overlap);
        for (int k = 0; k < ns; ++k)
            for (int64_t z : z1) zs.push_back(k * sd + z);
    }
    const auto ys = tile_starts(dy, ty_, overlap), xs = tile_starts(dx, tx_, overlap);
    const int64_t total = static_cast<int64_t>(zs.size()) * ys.size() * xs.size();
    if (tile_end < 0 || tile_end > total) tile_end = total;
    if (tile_begin < 0) tile_begin = 0;
    if (tile_begin >= tile_end) return ok();
    // the output crop (src/ml/infer.hpp:462-472): origin clamped into the volume, extent to its end
    const int64_t dims[3] = {full_dz, dy, dx};
    int64_t co[3], ce[3];
    bool cropped = false;
    for (int a = 0; a < 3; ++a) {
        co[a] = std::clamp<int64_t>(ro.core_org[a], 0, dims[a]);
        ce[a] = ro.core_ext[a] <= 0 ? dims[a] - co[a] : std::min(ro.core_ext[a], dims[a] - co[a]);
        cropped |= co[a] != 0 || ce[a] != dims[a];
    }
    // TTA: every tile once per member (src/ml/infer.hpp:554)
    const int ne = tta <= 1 ? 1 : std::min(tta, fxk::kTtaMaxMembers);
    std::vector<fxk::TileOrigin> cand;  // slab-local origins of the tiles that run
    for (int64_t i = tile_begin; i < tile_end; ++i) {
        const int64_t xi = i % static_cast<int64_t>(xs.size());
        const int64_t yi = (i / static_cast<int64_t>(xs.size())) % static_cast<int64_t>(ys.size());
        const int64_t zi = i / (static_cast<int64_t>(xs.size()) * ys.size());
        const int64_t z0 = zs[zi], y0 = ys[yi], x0 = xs[xi];
        // a tile that does not reach the core contributes nothing (src/ml/infer.hpp:532-543)
        if (cropped && !(z0 < co[0] + ce[0] && z0 + tz_ > co[0] && y0 < co[1] + ce[1] && y0 + ty_ > co[1] &&
                         x0 < co[2] + ce[2] && x0 + tx_ > co[2]))
            continue;
        if (ro.filter && !ro.filter(z0, y0, x0, tz_, ro.filter_user)) continue;
        const int64_t zl = z0 - z_origin;  // slab-local
        if (zl < 0 || (zl + tz_ > dz && full_dz >= tz_))
            return fail(kInvalid, "predict: tile " + std::to_string(i) + " is outside the z-slab");
        cand.push_back({zl, y0, x0});
    }
    if (ro.skip_constant && !cand.empty()) {
        // tiles whose input voxels all hold one value are not run (src/ml/inference.cpp:1487-1496,
        // 1885-1900): exact Σ / Σ² per tile on the device, n Σ² == (Σ)² <=> constant
        const size_t nc = cand.size();
        auto* d_org = static_cast<fxk::TileOrigin*>(dalloc(sizeof(fxk::TileOrigin) * nc));
        auto* d_s = static_cast<unsigned long long*>(dalloc(sizeof(unsigned long long) * 2 * nc));
        auto* d_lut = static_cast<float*>(dalloc(sizeof(float) * 256 * nc));
        auto* d_flag = static_cast<uint8_t*>(dalloc(nc));
        if (!d_org || !d_s || !d_lut || !d_flag) return fail(kInternal, "cudaMalloc: constant-tile check");
        std::vector<uint8_t> flag(nc, 0);
        Status st = cuda_status(cudaMemcpyAsync(d_org, cand.data(), sizeof(fxk::TileOrigin) * nc, cudaMemcpyHostToDevice, s),
                                "H2D tiles");
        if (st.ok()) st = cuda_status(cudaMemsetAsync(d_s, 0, sizeof(unsigned long long) * 2 * nc, s), "memset");
        for (size_t i0 = 0; st.ok() && i0 < nc; i0 += 65535) {
            const int n = static_cast<int>(std::min<size_t>(65535, nc - i0));
            st = cuda_status(fxk::launch_tile_sums(d_vol, dz, dy, dx, d_org + i0, n, tile(), d_s + 2 * i0, s), "tile_sums");
            if (st.ok())
                st = cuda_status(fxk::launch_tile_lut(d_s + 2 * i0, nullptr, n, tile().count(), 2,
                                                      d_lut + 256 * i0, d_flag + i0, s),
                                 "tile_lut");
        }
        if (st.ok()) st = cuda_status(cudaMemcpyAsync(flag.data(), d_flag, nc, cudaMemcpyDeviceToHost, s), "D2H flags");
        if (st.ok()) st = cuda_status(cudaStreamSynchronize(s), "constant-tile check");
        for (void* p : {static_cast<void*>(d_org), static_cast<void*>(d_s), static_cast<void*>(d_lut), static_cast<void*>(d_flag)}) {
            cudaFree(p);
            allocs_.erase(std::remove(allocs_.begin(), allocs_.end(), p), allocs_.end());
        }
        if (!st.ok()) return st;
        size_t k = 0;
        for (size_t i = 0; i < nc; ++i)
            if (!flag[i]) cand[k++] = cand[i];
        cand.resize(k);
    }
    std::vector<fxk::TileOrigin> tiles;
    std::vector<uint8_t> members;
    tiles.reserve(cand.size() * ne);
    for (const auto& t : cand)
        for (int m = 0; m < ne; ++m) {
            tiles.push_back(t);
            members.push_back(static_cast<uint8_t>(m));
        }
    if (tiles.empty()) return ok();
    if (static_cast<int64_t>(tiles.size()) > d_tiles_cap_) {
        void* p = dalloc(sizeof(fxk::TileOrigin) * tiles.size());
        void* q = dalloc(tiles.size());
        if (!p || !q) return fail(kInternal, "cudaMalloc: tile list");
        d_tiles_ = static_cast<fxk::TileOrigin*>(p);
        d_tta_ = static_cast<uint8_t*>(q);
        d_tiles_cap_ = static_cast<int64_t>(tiles.size());
    }
    Status st = cuda_status(cudaMemcpyAsync(d_tiles_, tiles.data(), sizeof(fxk::TileOrigin) * tiles.size(),
                                            cudaMemcpyHostToDevice, s),
                            "H2D tiles");
    if (!st.ok()) return st;
    if (ne > 1 && (st = cuda_status(cudaMemcpyAsync(d_tta_, members.data(), members.size(), cudaMemcpyHostToDevice, s),
                                    "H2D tta"))
                      .code)
        return st;
    // the accumulator window along y and x (the crop) for the head kernel
    norm_ = ro.norm;
    acc_y_shift_ = cropped ? -co[1] : 0;
    acc_dy_ = cropped ? ce[1] : 0;
    acc_x_shift_ = cropped ? -co[2] : 0;
    acc_dx_ = cropped ? ce[2] : 0;
    for (size_t i0 = 0; i0 < tiles.size(); i0 += batch) {
        const int nb = static_cast<int>(std::min<size_t>(batch, tiles.size() - i0));
        // accumulator window: acc plane 0 is volume plane acc_z_origin (default: the slab's origin)
        const int64_t shift = acc_dz < 0 ? 0 : z_origin - acc_z_origin;
        if ((st = forward(d_vol, dz, dy, dx, d_tiles_ + i0, nb, channel, sigmoid, d_acc, nullptr, false, s, shift,
                          acc_dz, ne > 1 ? d_tta_ + i0 : nullptr, 1.f / static_cast<float>(ne)))
                .code)
            break;
    }
    acc_y_shift_ = acc_dy_ = acc_x_shift_ = acc_dx_ = 0;
    return st;
}

}  // namespace fxh
