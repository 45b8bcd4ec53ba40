// fenix_b200/ml/ml_api.hpp — the stage-level drop-in of the B200 surface-prediction path: the
// reference's torch-free ML entry points (src/ml/ml_api.hpp:16-24) and their stage registration
// (src/ml/ml.hpp:22-42, registry src/core/core.hpp:68-108), over the C ABI of fenix_b200.h.
//   predict-surface <in.fxvol> <weights.fxweights> <out.fxvol> [patch] [overlap] [tta] [batch] [k=v]
//       run_predict_core (src/ml/inference.cpp:238-360, 362-740): the u8 archive's LOD 0 through the
//       net, the u8 prediction written as an archive at q = 32 (FENIX_PREDICT_Q overrides).
//   predict-scroll <ct.fxvol> <level> <weights.fxweights> <out_pred.fxvol> [k=v ...]
//       the global (zero-waste) grid of src/ml/inference.cpp:1282-1669 over an archive: chunk rows
//       are decoded on the device as the tile rows reach them, tile rows are blended into the
//       device GlobalAccum window, and finalised chunk rows are encoded and written as the
//       finalise front passes them, so host and device memory stay bounded by a tile row.
//   predict-ink ...  the reference's DINO-guided ink net, not part of this path: Errc::unsupported.
// Keys this path adds to both argument grammars: precision=f16|bf16|fp8 and device=N. fp8 nets are
// calibrated (scales and precision schedule) on four patches of the input.
#pragma once

#include "fenix_b200/codec/archive.hpp"
#include "fenix_b200/ml/infer.hpp"

#include <cstdlib>
#include <deque>
#include <functional>
#include <map>
#include <optional>
#include <span>
#include <string>
#include <string_view>
#include <vector>

namespace fenix_b200 {

// The reference's stage context (src/core/core.hpp:57-63).
struct Context {
    int threads = 0;
    bool cancelled = false;
    std::string project_dir;
};

// A stage = a CLI subcommand (src/core/core.hpp:68-108): registered once by name at static init.
struct Stage {
    std::string_view name;
    std::string_view help;
    std::function<Expected<int>(std::span<const std::string_view> args, Context&)> run;
};

inline std::vector<Stage>& registry() {
    static std::vector<Stage> stages;
    return stages;
}

inline int register_stage(Stage s) {
    for (const auto& e : registry())
        if (e.name == s.name) return 0;
    registry().push_back(std::move(s));
    return 0;
}

inline const Stage* find_stage(std::string_view name) {
    for (const auto& s : registry())
        if (s.name == name) return &s;
    return nullptr;
}

}  // namespace fenix_b200

namespace fenix_b200::ml {

namespace detail {

// Four P^3 patches of the volume, edge-clamped, at tiles spread over its tile grid: the
// calibration set of an fp8 net.
inline std::vector<u8> calibration_patches(VolumeView<const u8> v, int P, double overlap, int n = 4) {
    const Extent3 d = v.dims();
    const auto zs = fenix::ml::tile_starts(d.z, P, overlap), ys = fenix::ml::tile_starts(d.y, P, overlap),
               xs = fenix::ml::tile_starts(d.x, P, overlap);
    const s64 total = static_cast<s64>(zs.size() * ys.size() * xs.size());
    const std::size_t pv = static_cast<std::size_t>(P) * P * P;
    std::vector<u8> out(pv * static_cast<std::size_t>(n));
    for (int k = 0; k < n; ++k) {
        const s64 t = (2 * k + 1) * total / (2 * n);
        const s64 z0 = zs[static_cast<std::size_t>(t / static_cast<s64>(ys.size() * xs.size()))];
        const s64 y0 = ys[static_cast<std::size_t>((t / static_cast<s64>(xs.size())) % static_cast<s64>(ys.size()))];
        const s64 x0 = xs[static_cast<std::size_t>(t % static_cast<s64>(xs.size()))];
        u8* p = out.data() + pv * static_cast<std::size_t>(k);
        for (s64 z = 0; z < P; ++z)
            for (s64 y = 0; y < P; ++y)
                for (s64 x = 0; x < P; ++x)
                    *p++ = v(std::min(z0 + z, d.z - 1), std::min(y0 + y, d.y - 1), std::min(x0 + x, d.x - 1));
    }
    return out;
}

// fp8: per-tensor scales and the calibrated precision schedule (Dice >= 0.993 against the net's
// 16-bit forward on the calibration patches).
inline Expected<void> calibrate_fp8(B200Net& net, std::span<const u8> patches, int n) {
    if (auto r = net.calibrate(patches, n); !r) return r;
    double dice = 0, mx = 0;
    const fx_status st = fx_net_calibrate_schedule(net.handle(), patches.data(), n, 0.993, 0.0, &dice, &mx);
    if (st != FX_OK) return err_status(st, "calibrate_fp8");
    return {};
}

// The activation scales and per-layer precision schedule of a calibrated fp8 net, onto another
// replica of the same weights.
inline Expected<void> copy_fp8_state(const B200Net& from, B200Net& to) {
    std::vector<float> sc(1024);
    const int ns = fx_net_act_scales(from.handle(), sc.data(), static_cast<int>(sc.size()));
    std::vector<int> pr(1024);
    const int np = fx_net_layer_precision(from.handle(), pr.data(), nullptr, static_cast<int>(pr.size()));
    if (ns < 0 || ns > static_cast<int>(sc.size()) || np < 0 || np > static_cast<int>(pr.size()))
        return err(Errc::internal, "copy_fp8_state: too many layers");
    fx_status st = fx_net_set_act_scales(to.handle(), sc.data(), ns);
    if (st == FX_OK) st = fx_net_set_layer_precision(to.handle(), pr.data(), np);
    if (st != FX_OK) return err_status(st, "copy_fp8_state");
    return {};
}

inline float predict_q() {
    const char* e = std::getenv("FENIX_PREDICT_Q");
    const float q = e ? static_cast<float>(std::atof(e)) : 0.0f;
    return q > 0.0f ? q : 32.0f;
}

}  // namespace detail

// predict-surface (src/ml/inference.cpp:721-740 -> run_predict 362-714 -> run_predict_core 238-360).
namespace detail {
// run_predict (src/ml/inference.cpp:362-714) over the C ABI: the stage's options after the
// argument grammar, the net, .fxvol in and out.
[[nodiscard]] inline Expected<int> run_predict(std::span<const std::string_view> args, std::string_view name,
                                               void (*stage_defaults)(InferOptions&)) {
    auto a = parse_predict_args(args, name);
    if (!a) return std::unexpected(a.error());
    if (stage_defaults) stage_defaults(a->opt);
    if (!a->batch_explicit) a->opt.batch = 8;
    if (!a->opt.ckpt_path.empty()) {  // the checkpoint's identity, as the reference computes it
        a->opt.weights_hash = weights_hash64(a->weights);
        a->opt.input_hash = hash64({reinterpret_cast<const u8*>(a->in.data()), a->in.size()});
    }
    auto in = codec::VolumeArchive::open(a->in, a->device);
    if (!in) return std::unexpected(in.error());
    if (in->src_dtype() != codec::DType::u8)
        return err(Errc::unsupported, std::string(name) + ": the input archive is not u8");
    auto net = B200Net::load(a->weights, a->opt.patch, a->opt.batch, a->precision, a->device);
    if (!net) return std::unexpected(net.error());
    auto fx_norm_of = [](Norm n) {
        return n == Norm::pct_minmax ? FX_NORM_PCT_MINMAX : (n == Norm::unit255 ? FX_NORM_UNIT255 : FX_NORM_ZSCORE);
    };
    if (fx_net_set_norm(net->handle(), fx_norm_of(a->opt.norm)) != FX_OK)  // calibration sees the stage's inputs
        return err(Errc::internal, std::string(name) + ": fx_net_set_norm");
    const float q = detail::predict_q();
    if (a->precision != Precision::fp8 && a->gpus == 1) {
        if (auto r = predict_surface_fxvol(*net, a->in, a->out, a->opt, q); !r) return std::unexpected(r.error());
        return 0;
    }
    auto vol = in->read_volume_u8();
    if (!vol) return std::unexpected(vol.error());
    const VolumeView<const u8> v = static_cast<const Volume<u8>&>(*vol).view();
    if (a->precision == Precision::fp8) {
        const auto cal = detail::calibration_patches(v, a->opt.patch, a->opt.overlap);
        if (auto r = detail::calibrate_fp8(*net, cal, 4); !r) return std::unexpected(r.error());
    }
    // gpus = N: replicas on devices [device, device + N) with net 0's scales and schedule
    std::vector<B200Net> more;
    std::vector<B200Net*> all{&*net};
    for (int g = 1; g < a->gpus; ++g) {
        auto m = B200Net::load(a->weights, a->opt.patch, a->opt.batch, a->precision, a->device + g);
        if (!m) return std::unexpected(m.error());
        fx_net_set_norm(m->handle(), fx_norm_of(a->opt.norm));
        if (a->precision == Precision::fp8)
            if (auto r = detail::copy_fp8_state(*net, *m); !r) return std::unexpected(r.error());
        more.push_back(std::move(*m));
    }
    for (B200Net& m : more) all.push_back(&m);
    auto pred = a->gpus == 1 ? predict_surface_u8(v, *net, a->opt) : predict_surface_multi_u8(v, all, a->opt);
    if (!pred) return std::unexpected(pred.error());
    auto out = codec::VolumeArchive::create(a->out, pred->dims(), {q}, codec::DType::u8, a->device);
    if (!out) return std::unexpected(out.error());
    if (auto r = out->write_volume(static_cast<const Volume<u8>&>(*pred).view()); !r) return std::unexpected(r.error());
    if (auto r = out->close(); !r) return std::unexpected(r.error());
    return 0;
}
}  // namespace detail

// predict-surface (src/ml/inference.cpp:721-740): the surface net, softmax channel 1, zscore.
[[nodiscard]] inline Expected<int> run_predict_surface(std::span<const std::string_view> args) {
    return detail::run_predict(args, "predict-surface", nullptr);
}

// predict-ink (src/ml/inference.cpp:898-908): the same driver with the ink net's options — one
// class through a sigmoid, percentile (0.5 / 99.5) min-max normalisation. The net is whatever the
// weights hold; the reference's ink checkpoints (nets::ResEncUNet with shared_decoder +
// task_heads.ink) load as residual UNets with a task head.
[[nodiscard]] inline Expected<int> run_predict_ink(std::span<const std::string_view> args) {
    return detail::run_predict(args, "predict-ink", [](InferOptions& o) {
        o.sigmoid = true;
        o.channel = 0;
        o.norm = Norm::pct_minmax;
    });
}

// predict-scroll, global mode over a u8 .fxvol (src/ml/inference.cpp:989-1669). net=ink takes the
// ink net's contract (src/ml/inference.cpp:1084-1099: sigmoid on channel 0, percentile min-max).
// Zarr / URL roots, region mode, occupancy and raw-CT side inputs are not part of this path and give
// Errc::unsupported; gpuworkers / ahead / commit are accepted (the device window replaces them).
[[nodiscard]] inline Expected<int> run_predict_scroll(std::span<const std::string_view> args) {
    if (args.size() < 4)
        return err(Errc::invalid_argument,
                   "usage: predict-scroll <ct.fxvol> <level> <weights.fxweights> <out_pred.fxvol> [tta=8] [batch=2] "
                   "[patch=256] [overlap=0.5] [q=32] [bbox=z0,y0,x0,D,H,W] [net=surface|ink] [precision=f16|bf16|fp8] "
                   "[device=N]");
    const std::string root(args[0]), wpath(args[2]), out_path(args[3]);
    if (root.size() < 6 || root.substr(root.size() - 6) != ".fxvol")
        return err(Errc::unsupported, "predict-scroll: only .fxvol inputs are read on the B200 path (zarr / URL roots are not)");
    if (args[1] != "0") return err(Errc::unsupported, "predict-scroll: level must be 0 (LOD 0 of the archive)");
    InferOptions opt;
    opt.tta = 8;
    opt.batch = 2;
    opt.patch = 256;
    opt.overlap = 0.5;
    float q = 32.0f;
    Precision prec = Precision::f16;
    int device = 0;
    s64 bb[6] = {0, 0, 0, -1, -1, -1};
    auto num = [](std::string_view v, auto& out) -> bool {
        const auto r = std::from_chars(v.data(), v.data() + v.size(), out);
        return r.ec == std::errc{} && r.ptr == v.data() + v.size();
    };
    for (std::size_t i = 4; i < args.size(); ++i) {
        const std::string_view t = args[i];
        const auto eq = t.find('=');
        if (eq == std::string_view::npos) return err(Errc::invalid_argument, "predict-scroll: unknown arg '" + std::string(t) + "'");
        const std::string_view k = t.substr(0, eq), v = t.substr(eq + 1);
        bool ok = true;
        if (k == "tta") ok = num(v, opt.tta);
        else if (k == "batch") ok = num(v, opt.batch);
        else if (k == "patch") ok = num(v, opt.patch);
        else if (k == "overlap") ok = num(v, opt.overlap);
        else if (k == "q") ok = num(v, q);
        else if (k == "device") ok = num(v, device);
        else if (k == "bbox") {
            std::size_t p = 0;
            for (int j = 0; j < 6 && ok; ++j) {
                const std::size_t c = v.find(',', p);
                ok = num(v.substr(p, c == std::string_view::npos ? std::string_view::npos : c - p), bb[j]);
                p = c == std::string_view::npos ? v.size() : c + 1;
                if (j < 5 && c == std::string_view::npos) ok = false;
            }
        } else if (k == "precision") {
            if (v == "f16" || v == "half") prec = Precision::f16;
            else if (v == "bf16") prec = Precision::bf16;
            else if (v == "fp8") prec = Precision::fp8;
            else ok = false;
        } else if (k == "mode") {
            if (v != "global") return err(Errc::unsupported, "predict-scroll: only mode=global runs on the B200 path");
        } else if (k == "net") {
            if (v == "ink") {
                opt.sigmoid = true;
                opt.channel = 0;
                opt.norm = Norm::pct_minmax;
            } else if (v == "surface") {
                opt.sigmoid = false;
                opt.channel = 1;
                opt.norm = Norm::zscore;
            } else {
                return err(Errc::invalid_argument, "predict-scroll: net must be surface or ink");
            }
        } else if (k == "gpuworkers" || k == "ahead" || k == "commit") {
            // replicas per device, lookahead rows and commit cadence: the device window replaces them
        } else if (k == "ct" || k == "occ" || k == "ctq" || k == "halo" || k == "region") {
            return err(Errc::unsupported, "predict-scroll: " + std::string(k) + "= is not part of the B200 path");
        } else {
            return err(Errc::invalid_argument, "predict-scroll: unknown arg '" + std::string(t) + "'");
        }
        if (!ok) return err(Errc::invalid_argument, "predict-scroll: bad value in '" + std::string(t) + "'");
    }
    auto in = codec::VolumeArchive::open(root, device);
    if (!in) return std::unexpected(in.error());
    if (in->src_dtype() != codec::DType::u8) return err(Errc::unsupported, "predict-scroll: the input archive is not u8");
    const Extent3 D = in->dims();
    const codec::DctParams ip = in->params();
    // the bbox, widened to whole 64^3 chunks (the global grid's chunk-aligned origin)
    constexpr s64 T = 64;
    const s64 full[3] = {D.z, D.y, D.x};
    s64 org[3], ext[3];
    for (int j = 0; j < 3; ++j) {
        const s64 lo = std::clamp<s64>(bb[j], 0, full[j]);
        const s64 hi = bb[3 + j] < 0 ? full[j] : std::min(full[j], lo + bb[3 + j]);
        org[j] = lo / T * T;
        ext[j] = hi - org[j];
        if (ext[j] < 1) return err(Errc::invalid_argument, "predict-scroll: empty bbox");
    }
    auto net = B200Net::load(wpath, opt.patch, opt.batch, prec, device);
    if (!net) return std::unexpected(net.error());
    if (opt.batch > net->batch()) opt.batch = net->batch();
    if (fx_net_set_norm(net->handle(), opt.norm == Norm::pct_minmax ? FX_NORM_PCT_MINMAX : FX_NORM_ZSCORE) != FX_OK)
        return err(Errc::internal, "predict-scroll: fx_net_set_norm");
    auto acc = GlobalAccum::create({org[0], org[1], org[2]}, {ext[0], ext[1], ext[2]}, opt.patch, opt.overlap, 0, device);
    if (!acc) return std::unexpected(acc.error());
    auto out = codec::VolumeArchive::create(out_path, D, {q}, codec::DType::u8, device);
    if (!out) return std::unexpected(out.error());
    // decoded chunk rows of the bbox's y / x chunks, by chunk row index (archive coordinates)
    const s64 cy0 = org[1] / T, cy1 = (org[1] + ext[1] + T - 1) / T, cx0 = org[2] / T, cx1 = (org[2] + ext[2] + T - 1) / T;
    const s64 ny = cy1 - cy0, nx = cx1 - cx0, row_w = nx * T, row_plane = ny * T * row_w;
    std::map<s64, std::vector<u8>> rows;
    auto chunk_row = [&](s64 cz) -> Expected<const std::vector<u8>*> {
        if (auto it = rows.find(cz); it != rows.end()) return &it->second;
        std::vector<u8> slab(static_cast<std::size_t>(T * row_plane), 0);
        std::vector<u8> blob;
        std::vector<uint64_t> offs;
        std::vector<uint32_t> lens;
        std::vector<std::pair<s64, s64>> where;
        for (s64 cy = cy0; cy < cy1; ++cy)
            for (s64 cx = cx0; cx < cx1; ++cx) {
                if (in->coverage(0, {cz, cy, cx}) != codec::Coverage::Real) continue;  // ZERO / ABSENT: zeros
                auto p = in->chunk_payload(0, {cz, cy, cx});
                if (!p) return std::unexpected(p.error());
                offs.push_back(blob.size());
                lens.push_back(static_cast<uint32_t>(p->size()));
                blob.insert(blob.end(), p->begin(), p->end());
                where.push_back({cy - cy0, cx - cx0});
            }
        if (!where.empty()) {
            std::vector<u8> tiles(where.size() * static_cast<std::size_t>(T * T * T));
            const fx_status st = fx_fxvol_decode_tiles(blob.data(), blob.size(), offs.data(), lens.data(),
                                                       static_cast<int64_t>(where.size()), ip.q, ip.hf_exp, ip.dz_frac,
                                                       device, tiles.data(), nullptr);
            if (st != FX_OK) return err_status(st, "predict-scroll: chunk decode");
            for (std::size_t k = 0; k < where.size(); ++k)
                for (s64 z = 0; z < T; ++z)
                    for (s64 y = 0; y < T; ++y)
                        std::memcpy(slab.data() + z * row_plane + (where[k].first * T + y) * row_w + where[k].second * T,
                                    tiles.data() + k * T * T * T + (z * T + y) * T, static_cast<std::size_t>(T));
        }
        return &rows.emplace(cz, std::move(slab)).first->second;
    };
    // finalised chunks: encoded on the device in batches and written (all-zero chunks as ZERO)
    std::vector<ChunkCoord> pend;
    std::vector<u8> pend_u8;
    auto flush = [&]() -> Expected<void> {
        if (pend.empty()) return {};
        const std::size_t n = pend.size(), cv = static_cast<std::size_t>(T * T * T);
        std::vector<u8> enc(n * (cv + 4096));
        std::vector<uint64_t> offs(n);
        std::vector<uint32_t> lens(n);
        const fx_status st = fx_fxvol_encode_tiles(pend_u8.data(), nullptr, static_cast<int64_t>(n), q, 0.65f, 0.80f, device,
                                                   enc.data(), enc.size(), offs.data(), lens.data());
        if (st != FX_OK) return err_status(st, "predict-scroll: chunk encode");
        for (std::size_t k = 0; k < n; ++k) {
            const u8* c = pend_u8.data() + k * cv;
            const bool zero = std::all_of(c, c + cv, [](u8 v) { return v == 0; });
            auto r = out->write_chunk_payload(0, pend[k], zero ? std::span<const u8>() : std::span<const u8>(enc.data() + offs[k], lens[k]));
            if (!r) return r;
        }
        pend.clear();
        pend_u8.clear();
        return {};
    };
    auto sink = [&](ChunkCoord c, const u8* blk) {
        pend.push_back(c);
        pend_u8.insert(pend_u8.end(), blk, blk + T * T * T);
    };
    const s64 P = opt.patch, nrows = acc->tile_rows();
    std::vector<u8> planes;
    for (s64 zi = 0; zi < nrows; ++zi) {
        const s64 rs = acc->row_start(zi), re = std::min(rs + P, ext[0]);
        // chunk rows below this tile row are final once every earlier tile row is in
        if (auto r = acc->finalize_rows_below(rs / T, sink); !r) return std::unexpected(r.error());
        if (auto r = flush(); !r) return std::unexpected(r.error());
        planes.assign(static_cast<std::size_t>((re - rs) * ext[1] * ext[2]), 0);
        for (s64 z = rs; z < re; ++z) {
            const s64 az = org[0] + z;
            auto cr = chunk_row(az / T);
            if (!cr) return std::unexpected(cr.error());
            const u8* src = (*cr)->data() + (az % T) * row_plane;
            for (s64 y = 0; y < ext[1]; ++y)
                std::memcpy(planes.data() + ((z - rs) * ext[1] + y) * ext[2], src + (org[1] + y - cy0 * T) * row_w + (org[2] - cx0 * T),
                            static_cast<std::size_t>(ext[2]));
        }
        for (auto it = rows.begin(); it != rows.end();)  // chunk rows no later tile row reads
            it = it->first < (org[0] + rs) / T ? rows.erase(it) : std::next(it);
        if (prec == Precision::fp8 && zi == 0) {
            // calibration patches from the first tile row (edge-clamped)
            const VolumeView<const u8> v(planes.data(), {re - rs, ext[1], ext[2]});
            const auto cal = detail::calibration_patches(v, static_cast<int>(P), opt.overlap);
            if (auto r = detail::calibrate_fp8(*net, cal, 4); !r) return std::unexpected(r.error());
        }
        if (auto r = acc->predict_row(*net, zi, planes.data(), opt); !r) return std::unexpected(r.error());
    }
    if (auto r = acc->finalize_rows_below(acc->chunk_rows(), sink); !r) return std::unexpected(r.error());
    if (auto r = flush(); !r) return std::unexpected(r.error());
    if (auto r = out->set_nlods(1); !r) return std::unexpected(r.error());
    if (auto r = out->close(); !r) return std::unexpected(r.error());
    return 0;
}

}  // namespace fenix_b200::ml

// Stage registration (src/ml/ml.hpp:22-42): the same names and help lines as the reference's.
namespace fenix_b200::detail {
inline const int stage_predict_surface = ::fenix_b200::register_stage(::fenix_b200::Stage{
    "predict-surface", "surface-prediction inference (3D UNet, B200)",
    [](std::span<const std::string_view> a, ::fenix_b200::Context&) { return ::fenix_b200::ml::run_predict_surface(a); }});
inline const int stage_predict_scroll = ::fenix_b200::register_stage(::fenix_b200::Stage{
    "predict-scroll", "whole-scroll surface prediction (out-of-core, device-resident accumulator) -> .fxvol",
    [](std::span<const std::string_view> a, ::fenix_b200::Context&) { return ::fenix_b200::ml::run_predict_scroll(a); }});
inline const int stage_predict_ink = ::fenix_b200::register_stage(::fenix_b200::Stage{
    "predict-ink", "ink-detection inference over a u8 .fxvol (sigmoid, percentile normalisation) -> .fxvol",
    [](std::span<const std::string_view> a, ::fenix_b200::Context&) { return ::fenix_b200::ml::run_predict_ink(a); }});
}  // namespace fenix_b200::detail
