// ref_infer.cpp — runs the REFERENCE's own CPU inference path on a dense u8 volume, so the
// oracle and the GPU path can be compared with what the reference itself computes. Oracle
// tooling (test infrastructure), compiled from the reference sources by oracle/Makefile into
// oracle/_ref/; not product code.
//
// The net is the plain nnU-Net UNet composed from the reference's own modules:
// nets::ConvStack (src/ml/nets/resenc_unet.hpp:141-158) per encoder/decoder stage,
// nn::ConvTranspose3d(2, s2) upsampling and the nn::Conv3d 1x1x1 head, wired as
// DecoderImpl::forward does (resenc_unet.hpp:227-237) with `nconv` convs per decoder stage.
// Weights come through the reference's load_fxweights + load_into (src/ml/weights.hpp), the
// driver is ml::predict_surface_filled (src/ml/infer.hpp:456-864) with half=false (fp32 on
// CPU), fed by a dense u8 filler with edge clamp as run_predict_core uses
// (src/ml/inference.cpp:309-321).
//
// usage: ref_infer <w.fxweights> <vol.u8> dz dy dx patch overlap batch <out.f32|-> [threads] [key=value ...]
//   keys (InferOptions fields, src/ml/infer.hpp:38-103): tta=N, norm=zscore|pct_minmax|unit255,
//   channel=N, sigmoid=0|1, core=z,y,x,dz,dy,dx (output crop), skipconst=1 (the constant-input tile
//   filter of predict-scroll's region mode, src/ml/inference.cpp:1885-1900), ckpt=<path> with
//   whash=<u64> ihash=<u64> (InferOptions::ckpt_path / weights_hash / input_hash), stopafter=K (the
//   filler fails on its (K+1)-th patch: the reference then saves its progress to ckpt and exits 1,
//   src/ml/infer.hpp:840-846 — the run a resume continues)
// prints one JSON line: {"seconds": ..., "threads": ..., "tiles": ..., "dims": [z, y, x]} and writes the
// f32 probability volume (the core's dims when cropped).
#include "ml/infer.hpp"
#include "ml/weights.hpp"

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <vector>

namespace nets = fenix::ml::nets;
namespace nn = torch::nn;
using namespace fenix;

struct EncImpl : nn::Module {
    nn::ModuleList stages{nullptr};
    std::vector<nets::ConvStack> st;
    EncImpl(const std::vector<int>& f, int nconv) {
        stages = nn::ModuleList();
        int prev = 1;
        for (size_t s = 0; s < f.size(); ++s) {
            auto c = nets::ConvStack(prev, f[s], 3, s ? 2 : 1, nconv);
            st.push_back(c);
            stages->push_back(c);
            prev = f[s];
        }
        register_module("stages", stages);
    }
};
TORCH_MODULE(Enc);

struct DecImpl : nn::Module {
    nn::ModuleList transpconvs{nullptr}, stages{nullptr}, seg_layers{nullptr};
    std::vector<nn::ConvTranspose3d> tp;
    std::vector<nets::ConvStack> dec;
    std::vector<nn::Conv3d> seg;
    DecImpl(const std::vector<int>& f, int nconv, int ncls) {
        transpconvs = nn::ModuleList();
        stages = nn::ModuleList();
        seg_layers = nn::ModuleList();
        const int n = static_cast<int>(f.size());
        for (int s = 0; s < n - 1; ++s) {
            const int below = f[n - 1 - s], skipc = f[n - 2 - s];
            auto t = nn::ConvTranspose3d(nn::ConvTranspose3dOptions(below, skipc, 2).stride(2).bias(true));
            tp.push_back(t);
            transpconvs->push_back(t);
            auto c = nets::ConvStack(2 * skipc, skipc, 3, 1, nconv);
            dec.push_back(c);
            stages->push_back(c);
            auto sl = nn::Conv3d(nn::Conv3dOptions(skipc, ncls, 1).bias(true));
            seg.push_back(sl);
            seg_layers->push_back(sl);
        }
        register_module("transpconvs", transpconvs);
        register_module("stages", stages);
        register_module("seg_layers", seg_layers);
    }
};
TORCH_MODULE(Dec);

struct PlainImpl : nn::Module {
    Enc encoder{nullptr};
    Dec decoder{nullptr};
    PlainImpl(const std::vector<int>& f, int nconv, int ncls) {
        encoder = register_module("encoder", Enc(f, nconv));
        decoder = register_module("decoder", Dec(f, nconv, ncls));
    }
    torch::Tensor forward(torch::Tensor x) {
        std::vector<torch::Tensor> skips;
        for (auto& s : encoder->st) {
            x = s(x);
            skips.push_back(x);
        }
        const int n = static_cast<int>(skips.size());
        torch::Tensor lres = skips.back();
        for (size_t s = 0; s < decoder->tp.size(); ++s) {
            torch::Tensor u = decoder->tp[s]->forward(lres);
            u = torch::cat({u, skips[n - 2 - static_cast<int>(s)]}, 1);
            lres = decoder->dec[s](u);
        }
        return decoder->seg.back()->forward(lres);
    }
};
TORCH_MODULE(Plain);

// Run the reference's predict_surface_filled with `net` on the volume file and write the result.
template <class Net>
int run(Net& net, int argc, char** argv, Extent3 d, const std::string& vpath, const std::string& opath) {
    Volume<u8> vol(d);
    {
        std::FILE* fp = std::fopen(vpath.c_str(), "rb");
        if (!fp || std::fread(vol.data(), 1, static_cast<size_t>(d.count()), fp) != static_cast<size_t>(d.count())) {
            std::fprintf(stderr, "cannot read %s\n", vpath.c_str());
            return 1;
        }
        std::fclose(fp);
    }
    ml::InferOptions opt;
    opt.patch = std::atoi(argv[6]);
    opt.overlap = std::atof(argv[7]);
    opt.batch = std::atoi(argv[8]);
    opt.half = false;  // fp32 on the CPU
    const VolumeView<const u8> uv = vol.view();
    long stop_after = -1;
    for (int i = 10; i < argc; ++i) {
        const std::string a = argv[i];
        const auto eq = a.find('=');
        if (eq == std::string::npos) continue;  // the positional thread count
        const std::string k = a.substr(0, eq), v = a.substr(eq + 1);
        if (k == "tta") opt.tta = std::atoi(v.c_str());
        else if (k == "channel") opt.channel = std::atoi(v.c_str());
        else if (k == "sigmoid") opt.sigmoid = std::atoi(v.c_str()) != 0;
        else if (k == "norm") opt.norm = v == "pct_minmax" ? ml::Norm::pct_minmax : (v == "unit255" ? ml::Norm::unit255 : ml::Norm::zscore);
        else if (k == "core") {
            long long c[6] = {0, 0, 0, -1, -1, -1};
            std::sscanf(v.c_str(), "%lld,%lld,%lld,%lld,%lld,%lld", &c[0], &c[1], &c[2], &c[3], &c[4], &c[5]);
            opt.core_org = {c[0], c[1], c[2]};
            opt.core_ext = {c[3], c[4], c[5]};
        } else if (k == "ckpt") {
            opt.ckpt_path = v;
        } else if (k == "whash") {
            opt.weights_hash = std::strtoull(v.c_str(), nullptr, 10);
        } else if (k == "ihash") {
            opt.input_hash = std::strtoull(v.c_str(), nullptr, 10);
        } else if (k == "stopafter") {
            stop_after = std::atol(v.c_str());
        } else if (k == "skipconst" && v == "1") {
            opt.tile_filter = [uv](s64 z0, s64 y0, s64 x0, s64 P) {
                const Extent3 dd = uv.dims();
                const s64 z1 = std::min(dd.z, z0 + P), y1 = std::min(dd.y, y0 + P), x1 = std::min(dd.x, x0 + P);
                const u8 first = uv(std::min(z0, dd.z - 1), std::min(y0, dd.y - 1), std::min(x0, dd.x - 1));
                for (s64 z = z0; z < z1; ++z)
                    for (s64 y = y0; y < y1; ++y)
                        for (s64 x = x0; x < x1; ++x)
                            if (uv(z, y, x) != first) return true;
                return false;
            };
        }
    }
    const auto t0 = std::chrono::steady_clock::now();
    long filled = 0;
    auto prob = ml::predict_surface_filled(
        d,
        [uv, stop_after, &filled](s64 z0, s64 y0, s64 x0, int P, float* out) {
            if (stop_after >= 0 && filled++ >= stop_after) throw std::runtime_error("stopafter: filler stops");
            parallel_for(0, P, [&](s64 z) {
                for (int y = 0; y < P; ++y)
                    for (int x = 0; x < P; ++x)
                        out[(static_cast<std::size_t>(z) * P + y) * P + x] =
                            static_cast<f32>(uv.at_clamped(z0 + z, y0 + y, x0 + x));
            });
        },
        net, torch::Device(torch::kCPU), opt);
    const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (!prob) {
        std::fprintf(stderr, "predict: %s\n", prob.error().message.c_str());
        return 1;
    }
    const Extent3 od = prob->dims();
    if (opath != "-") {
        std::FILE* fp = std::fopen(opath.c_str(), "wb");
        if (!fp) return 1;
        std::fwrite(prob->data(), sizeof(float), static_cast<size_t>(od.count()), fp);
        std::fclose(fp);
    }
    const long tiles = static_cast<long>(ml::tile_starts(d.z, opt.patch, opt.overlap).size() *
                                         ml::tile_starts(d.y, opt.patch, opt.overlap).size() *
                                         ml::tile_starts(d.x, opt.patch, opt.overlap).size());
    std::printf("{\"seconds\": %.6f, \"threads\": %d, \"tiles\": %ld, \"dims\": [%lld, %lld, %lld]}\n", dt,
                torch::get_num_threads(), tiles, static_cast<long long>(od.z), static_cast<long long>(od.y),
                static_cast<long long>(od.x));
    return 0;
}

int main(int argc, char** argv) {
    if (argc < 10) {
        std::fprintf(stderr, "usage: ref_infer <w.fxweights> <vol.u8> dz dy dx patch overlap batch <out.f32|-> [threads]\n");
        return 2;
    }
    const std::string wpath = argv[1], vpath = argv[2], opath = argv[9];
    const Extent3 d{std::atoll(argv[3]), std::atoll(argv[4]), std::atoll(argv[5])};
    if (argc > 10 && std::string(argv[10]).find('=') == std::string::npos) torch::set_num_threads(std::atoi(argv[10]));
    auto wm = ml::load_fxweights(wpath);
    if (!wm) {
        std::fprintf(stderr, "load_fxweights: %s\n", wm.error().message.c_str());
        return 1;
    }
    // residual-encoder UNet (the reference's own nets::ResEncUNet): stem + blocks in the weights
    for (const std::string enc : {"encoder", "shared_encoder"}) {
        if (!wm->count(enc + ".stem.convs.0.conv.weight")) continue;
        nets::ResEncUNetConfig cfg;
        cfg.plain_naming = enc == "encoder";
        cfg.features.clear();
        cfg.blocks.clear();
        cfg.strides.clear();
        for (int s = 0;; ++s) {
            const std::string st = enc + ".stages." + std::to_string(s) + ".blocks.";
            if (!wm->count(st + "0.conv1.conv.weight")) break;
            cfg.features.push_back(static_cast<int>(wm->at(st + "0.conv1.conv.weight").size(0)));
            int nb = 0;
            while (wm->count(st + std::to_string(nb) + ".conv1.conv.weight")) ++nb;
            cfg.blocks.push_back(nb);
            cfg.strides.push_back(s ? 2 : 1);
        }
        cfg.squeeze_excitation = wm->count(enc + ".stages.0.blocks.0.squeeze_excitation.sSE.conv.weight") > 0;
        // ink checkpoints: shared_decoder + task_heads.<task> (the reference's predict-ink config,
        // src/ml/inference.cpp:898-908)
        cfg.task_head = wm->count("shared_decoder.transpconvs.0.weight") > 0;
        if (cfg.task_head) {
            for (const auto& kv : *wm)
                if (kv.first.rfind("task_heads.", 0) == 0 && kv.first.size() > 7 &&
                    kv.first.compare(kv.first.size() - 7, 7, ".weight") == 0)
                    cfg.task = kv.first.substr(11, kv.first.size() - 7 - 11);
            cfg.num_classes = static_cast<int>(wm->at("task_heads." + cfg.task + ".weight").size(0));
        } else {
            const std::string dec = cfg.plain_naming ? "decoder" : "task_decoders." + cfg.task;
            cfg.num_classes = static_cast<int>(
                wm->at(dec + ".seg_layers." + std::to_string(cfg.features.size() - 2) + ".weight").size(0));
        }
        nets::ResEncUNet rnet(cfg);
        rnet->eval();
        std::vector<std::string> miss;
        ml::load_into(*rnet, *wm, &miss);
        if (!miss.empty()) {
            std::fprintf(stderr, "weights missing %s\n", miss[0].c_str());
            return 1;
        }
        return run(rnet, argc, argv, d, vpath, opath);
    }
    std::vector<int> f;
    int nconv = 0;
    for (;;) {
        auto it = wm->find("encoder.stages." + std::to_string(f.size()) + ".convs.0.conv.weight");
        if (it == wm->end()) break;
        f.push_back(static_cast<int>(it->second.size(0)));
    }
    while (wm->count("encoder.stages.0.convs." + std::to_string(nconv) + ".conv.weight")) ++nconv;
    const int ncls = static_cast<int>(wm->at("decoder.seg_layers." + std::to_string(f.size() - 2) + ".weight").size(0));
    Plain net(f, nconv, ncls);
    net->eval();
    std::vector<std::string> missing;
    ml::load_into(*net, *wm, &missing);
    if (!missing.empty()) {
        std::fprintf(stderr, "weights missing %s\n", missing[0].c_str());
        return 1;
    }
    return run(net, argc, argv, d, vpath, opath);
}
