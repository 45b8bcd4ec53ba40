// Exercises the header-only host API (fenix_b200/ml/infer.hpp) against the C ABI.
//   host_api_test cpu                   — argument grammar, option checks, views, error mapping
//   host_api_test gpu <weights> <out>   — predict_surface_window and predict_surface_u8 on a
//                                         synthetic window; writes both outputs to <out>
//   host_api_test fxvol <in> <out>      — codec::VolumeArchive: open an archive, check its metadata
//                                         and rewrite every chunk payload of every LOD to <out>
//   host_api_test stages <weights> <dir> — the predict-surface / predict-scroll stages through the
//                                         registry on an archive written in <dir>, against
//                                         predict_surface_u8; predict_surface_filled, crops, filters
#include "fenix_b200/codec/archive.hpp"
#include "fenix_b200/ml/infer.hpp"
#include "fenix_b200/ml/ml_api.hpp"
#include "fenix_b200/ml/tiling.hpp"
#include "fenix_b200_synth.h"

#include <cmath>
#include <cstdio>
#include <fstream>
#include <vector>

using namespace fenix_b200;

static int fails = 0;
#define CHECK(c)                                                             \
    do {                                                                     \
        if (!(c)) {                                                          \
            std::fprintf(stderr, "%s:%d: CHECK failed: %s\n", __FILE__, __LINE__, #c); \
            ++fails;                                                         \
        }                                                                    \
    } while (0)

static Expected<ml::PredictArgs> parse(std::vector<std::string_view> v) { return ml::parse_predict_args(v); }

static int cpu() {
    {
        auto a = parse({"in.fxvol", "w.fxweights", "out.fxvol"});
        CHECK(a && a->opt.patch == 256 && a->opt.overlap == 0.5 && a->opt.batch == 3 && !a->batch_explicit);
    }
    {
        auto a = parse({"in", "w", "out", "128", "0.25", "0", "8"});
        CHECK(a && a->opt.patch == 128 && a->opt.overlap == 0.25 && a->opt.tta == 0 && a->opt.batch == 8 &&
              a->batch_explicit);
    }
    {  // a keyword token in a positional slot is skipped, not parsed as a number
        auto a = parse({"in", "w", "out", "precision=fp8", "0.5", "batch=4"});
        CHECK(a && a->precision == ml::Precision::fp8 && a->opt.batch == 4 && a->opt.patch == 256);
    }
    CHECK(!parse({"in", "w"}) && parse({"in", "w"}).error().code == Errc::invalid_argument);
    CHECK(parse({"in", "w", "out", "12x"}).error().code == Errc::invalid_argument);
    {  // positional tta: the octahedral members go to the ABI
        auto a = parse({"in", "w", "out", "128", "0.5", "8"});
        CHECK(a && a->opt.tta == 8 && ml::to_fx(a->opt) && ml::to_fx(a->opt)->tta == 8);
    }
    CHECK(parse({"in", "w", "out", "scales=0.8,1.0"}).error().code == Errc::unsupported);
    CHECK(parse({"in", "w", "out", "bogus=1"}).error().code == Errc::invalid_argument);
    CHECK(parse({"in", "w", "out", "precision=int4"}).error().code == Errc::invalid_argument);
    CHECK(parse({"in", "w", "out", "gpus=4"}) && parse({"in", "w", "out", "gpus=4"})->gpus == 4);
    CHECK(parse({"in", "w", "out", "gpus=0"}).error().code == Errc::invalid_argument);
    {
        auto a = parse({"in", "w", "out", "ckpt=/tmp/x.ckpt", "ckpt_every=64"});
        CHECK(a && a->opt.ckpt_path == "/tmp/x.ckpt" && a->opt.ckpt_every == 64);
        CHECK(a && ml::to_fx(a->opt) && std::string(ml::to_fx(a->opt)->ckpt_path) == "/tmp/x.ckpt");
    }
    {
        ml::InferOptions o;
        o.norm = ml::Norm::pct_minmax;
        CHECK(ml::to_fx(o) && ml::to_fx(o)->norm == FX_NORM_PCT_MINMAX);
        o = {};
        o.core_org = {8, 0, 4};
        o.core_ext = {64, -1, 32};
        auto c = ml::to_fx(o);
        CHECK(c && c->core_org[0] == 8 && c->core_org[2] == 4 && c->core_ext[0] == 64 && c->core_ext[1] == 0 &&
              c->core_ext[2] == 32);
        CHECK(ml::output_dims({100, 90, 80}, o) == (Extent3{64, 90, 32}));
        o.core_ext = {0, -1, -1};
        CHECK(ml::to_fx(o).error().code == Errc::invalid_argument);
        o = {};
        int seen = 0;
        o.tile_filter = [&](s64 z0, s64, s64, s64 P) { return ++seen, z0 + P > 100; };
        auto fo = ml::to_fx(o);
        CHECK(fo && fo->tile_filter && fo->tile_filter(64, 0, 0, 64, fo->tile_filter_user) == 1 &&
              fo->tile_filter(0, 0, 0, 64, fo->tile_filter_user) == 0 && seen == 2);
        o = {};
        o.overlap = 1.0;
        CHECK(ml::to_fx(o).error().code == Errc::invalid_argument);
        o = {};
        o.patch = 128;
        o.batch = 5;
        auto f = ml::to_fx(o);
        CHECK(f && f->patch == 128 && f->batch == 5 && f->channel == 1 && f->sigmoid == 0);
    }
    {  // strided views: a y-x transposed view reads the transposed element
        std::vector<u8> buf(2 * 3 * 4);
        for (std::size_t i = 0; i < buf.size(); ++i) buf[i] = static_cast<u8>(i);
        VolumeView<const u8> c(buf.data(), {2, 3, 4});
        CHECK(c.contiguous() && c(1, 2, 3) == 23);
        VolumeView<const u8> t(buf.data(), {2, 4, 3}, {12, 1, 4});
        CHECK(!t.contiguous() && t(1, 3, 2) == c(1, 2, 3));
        std::vector<u8> tmp;
        const u8* p = ml::detail::contiguous_input(t, tmp);
        CHECK(p == tmp.data() && tmp.size() == 24 && p[(1 * 4 + 3) * 3 + 2] == 23);
    }
    {  // errors carry the ABI status and message
        auto n = ml::B200Net::load("/nonexistent/w.fxweights", 64, 1);
        // not_found / io_error on a GPU machine; without a GPU the device check answers first
        CHECK(!n && n.error().code != Errc::ok && n.error().message.find("B200Net::load") != std::string::npos);
        ml::B200Net empty;
        std::vector<u8> v(8);
        auto r = ml::predict_surface_u8(VolumeView<const u8>(v.data(), {2, 2, 2}), empty, {});
        CHECK(!r && r.error().code == Errc::invalid_argument);
    }
    CHECK(static_cast<int>(Errc::internal) == FX_INTERNAL && static_cast<int>(Errc::unsupported) == FX_UNSUPPORTED);
    {  // the grid origin must be 64-aligned (checked before any device work)
        auto g = ml::GlobalAccum::create({32, 0, 0}, {128, 64, 64}, 64, 0.5);
        CHECK(!g && g.error().code == Errc::invalid_argument);
    }
    {  // the stage registry (src/core/core.hpp:68-108) holds the ML stages, idempotent by name
        CHECK(find_stage("predict-surface") && find_stage("predict-scroll") && find_stage("predict-ink"));
        CHECK(!find_stage("no-such-stage"));
        const std::size_t n = registry().size();
        register_stage(Stage{"predict-surface", "again", nullptr});
        CHECK(registry().size() == n);
        Context ctx;
        std::vector<std::string_view> a{"x"};
        auto r = find_stage("predict-ink")->run(a, ctx);
        CHECK(!r && r.error().code == Errc::invalid_argument);  // the predict grammar wants 3 arguments
        std::vector<std::string_view> z{"s3://bucket/scroll.zarr", "0", "w.fxweights", "out.fxvol"};
        r = find_stage("predict-scroll")->run(z, ctx);
        CHECK(!r && r.error().code == Errc::unsupported);
        std::vector<std::string_view> b{"ct.fxvol", "0", "w.fxweights", "out.fxvol", "bogus=1"};
        r = find_stage("predict-scroll")->run(b, ctx);
        CHECK(!r && r.error().code == Errc::invalid_argument);
        std::vector<std::string_view> nk{"ct.fxvol", "0", "w.fxweights", "out.fxvol", "net=dino"};
        r = find_stage("predict-scroll")->run(nk, ctx);
        CHECK(!r && r.error().code == Errc::invalid_argument);
        std::vector<std::string_view> m{"ct.fxvol", "0", "w.fxweights", "out.fxvol", "mode=region"};
        r = find_stage("predict-scroll")->run(m, ctx);
        CHECK(!r && r.error().code == Errc::unsupported);
        std::vector<std::string_view> u{"ct.fxvol"};
        r = find_stage("predict-surface")->run(u, ctx);
        CHECK(!r && r.error().code == Errc::invalid_argument);
    }
    std::printf("%s\n", fails ? "FAIL" : "ok");
    return fails ? 1 : 0;
}

// The stages over archives against the in-memory API on the same volume and net.
static int stages(const char* weights, const char* dir) {
    const Extent3 d{160, 96, 120};
    std::vector<u8> vol(static_cast<std::size_t>(d.count()));
    fx_spiral_params sp{12.0, 3.0, 170.0, 15.0, 40.0, 10.0, 1.0, 0.0};
    if (fx_synth_spiral(vol.data(), d.z, d.y, d.x, &sp, 9, 0, d.z) != 0) return 2;
    VolumeView<const u8> in(vol.data(), d);
    const std::string ip = std::string(dir) + "/in.fxvol", op = std::string(dir) + "/surf.fxvol",
                      sp2 = std::string(dir) + "/scroll.fxvol";
    {
        auto a = codec::VolumeArchive::create(ip, d, {8.0f});
        if (!a || !a->write_volume(in) || !a->close()) return 3;
    }
    auto src = codec::VolumeArchive::open(ip);
    if (!src) return 4;
    auto dec = src->read_volume_u8();  // what the stages see (the codec is lossy)
    if (!dec) return 5;
    const VolumeView<const u8> dv = static_cast<const Volume<u8>&>(*dec).view();
    Context ctx;
    {  // predict-surface: patch 64, overlap 0.5, no tta, batch 2
        std::vector<std::string_view> a{ip, weights, op, "64", "0.5", "0", "2"};
        auto r = find_stage("predict-surface")->run(a, ctx);
        if (!r) {
            std::fprintf(stderr, "predict-surface: %s\n", r.error().message.c_str());
            return 6;
        }
    }
    auto net = ml::B200Net::load(weights, 64, 2);
    if (!net) return 7;
    ml::InferOptions o;
    o.patch = 64;
    o.overlap = 0.5;
    o.batch = 2;
    auto want = ml::predict_surface_u8(dv, *net, o);
    if (!want) return 8;
    auto q32 = [&](const Volume<u8>& v) {  // what a q = 32 archive of v decodes to
        const std::string t = std::string(dir) + "/tmp.fxvol";
        auto a = codec::VolumeArchive::create(t, v.dims(), {32.0f});
        if (!a || !a->write_volume(v.view()) || !a->close()) return Volume<u8>{};
        auto b = codec::VolumeArchive::open(t);
        auto r = b ? b->read_volume_u8() : Expected<Volume<u8>>(std::unexpected(Error{}));
        return r ? std::move(*r) : Volume<u8>{};
    };
    auto got = codec::VolumeArchive::open(op);
    auto gv = got ? got->read_volume_u8() : Expected<Volume<u8>>(std::unexpected(Error{}));
    const Volume<u8> wq = q32(*want);
    CHECK(gv && wq.data() && std::memcmp(gv->data(), wq.data(), vol.size()) == 0);
    // predict-scroll writes each finalised chunk with the voxels past the volume at 0 (the
    // GlobalAccum sink), predict-surface's write_volume replicates the edge: encode an in-memory
    // prediction's chunks the scroll's way and compare the decoded results
    auto scroll_matches = [&](const Volume<u8>& want_v, const std::string& path, const char* label) -> bool {
        auto s2 = codec::VolumeArchive::open(path);
        auto sv = s2 ? s2->read_volume_u8() : Expected<Volume<u8>>(std::unexpected(Error{}));
        if (!sv) return false;
        const s64 T = 64, ncz = (d.z + T - 1) / T, ncy = (d.y + T - 1) / T, ncx = (d.x + T - 1) / T;
        const std::size_t n = static_cast<std::size_t>(ncz * ncy * ncx), cv = static_cast<std::size_t>(T * T * T);
        std::vector<u8> ch(n * cv, 0), enc(n * (cv + 4096)), dec(n * cv);
        std::vector<uint64_t> offs(n);
        std::vector<uint32_t> lens(n);
        for (s64 k = 0; k < static_cast<s64>(n); ++k) {
            const s64 cz = k / (ncy * ncx), cy = (k / ncx) % ncy, cx = k % ncx;
            for (s64 z = 0; z < T && cz * T + z < d.z; ++z)
                for (s64 y = 0; y < T && cy * T + y < d.y; ++y)
                    for (s64 x = 0; x < T && cx * T + x < d.x; ++x)
                        ch[k * cv + (z * T + y) * T + x] = want_v.data()[((cz * T + z) * d.y + cy * T + y) * d.x + cx * T + x];
        }
        if (fx_fxvol_encode_tiles(ch.data(), nullptr, static_cast<int64_t>(n), 32.0f, 0.65f, 0.80f, 0, enc.data(), enc.size(),
                                  offs.data(), lens.data()) != FX_OK ||
            fx_fxvol_decode_tiles(enc.data(), enc.size(), offs.data(), lens.data(), static_cast<int64_t>(n), 32.0f, 0.65f,
                                  0.80f, 0, dec.data(), nullptr) != FX_OK)
            return false;
        std::size_t far = 0;
        double sum = 0;
        for (s64 z = 0; z < d.z; ++z)
            for (s64 y = 0; y < d.y; ++y)
                for (s64 x = 0; x < d.x; ++x) {
                    const s64 k = ((z / T) * ncy + y / T) * ncx + x / T;
                    const int w0 = dec[k * cv + ((z % T) * T + y % T) * T + x % T];
                    const int dd = std::abs(int(sv->data()[(z * d.y + y) * d.x + x]) - w0);
                    sum += dd;
                    far += dd > 8;
                }
        std::fprintf(stderr, "%s (decoded q32): mean |d| %.4f, %zu voxels > 8\n", label,
                     sum / static_cast<double>(vol.size()), far);
        return sum / static_cast<double>(vol.size()) <= 0.25 && far * 1000 <= vol.size();
    };
    {  // predict-scroll over the same archive, global grid, no tta: the same tiles and blend
        std::vector<std::string_view> a{ip, "0", weights, sp2, "tta=0", "batch=2", "patch=64", "overlap=0.5"};
        auto r = find_stage("predict-scroll")->run(a, ctx);
        if (!r) {
            std::fprintf(stderr, "predict-scroll: %s\n", r.error().message.c_str());
            return 9;
        }
        CHECK(scroll_matches(*want, sp2, "predict-scroll vs predict_surface"));
    }
    {  // predict-ink: the same driver with sigmoid on channel 0 and percentile normalisation
        const std::string ik = std::string(dir) + "/ink.fxvol", sk = std::string(dir) + "/scroll_ink.fxvol";
        std::vector<std::string_view> a{ip, weights, ik, "64", "0.5", "0", "2"};
        auto r = find_stage("predict-ink")->run(a, ctx);
        if (!r) {
            std::fprintf(stderr, "predict-ink: %s\n", r.error().message.c_str());
            return 10;
        }
        ml::InferOptions io = o;
        io.sigmoid = true;
        io.channel = 0;
        io.norm = ml::Norm::pct_minmax;
        auto wi = ml::predict_surface_u8(dv, *net, io);
        auto gi = codec::VolumeArchive::open(ik);
        auto giv = gi ? gi->read_volume_u8() : Expected<Volume<u8>>(std::unexpected(Error{}));
        const Volume<u8> wiq = wi ? q32(*wi) : Volume<u8>{};
        CHECK(giv && wiq.data() && std::memcmp(giv->data(), wiq.data(), vol.size()) == 0);
        // and it differs from the surface stage's output (other channel, activation, normalisation)
        CHECK(giv && gv && std::memcmp(giv->data(), gv->data(), vol.size()) != 0);
        // predict-scroll net=ink: the ink contract over the global grid
        std::vector<std::string_view> b{ip, "0", weights, sk, "tta=0", "batch=2", "patch=64", "overlap=0.5", "net=ink"};
        r = find_stage("predict-scroll")->run(b, ctx);
        if (!r) {
            std::fprintf(stderr, "predict-scroll net=ink: %s\n", r.error().message.c_str());
            return 11;
        }
        CHECK(wi && scroll_matches(*wi, sk, "predict-scroll net=ink vs predict_surface (ink options)"));
    }
    {  // predict_surface_filled with a clamped filler = predict_surface on the dense view
        auto f = ml::predict_surface_filled(
            d,
            [&](s64 z0, s64 y0, s64 x0, int P, float* out) {
                for (s64 z = 0; z < P; ++z)
                    for (s64 y = 0; y < P; ++y)
                        for (s64 x = 0; x < P; ++x)
                            out[(z * P + y) * P + x] = in(std::min(z0 + z, d.z - 1), std::min(y0 + y, d.y - 1), std::min(x0 + x, d.x - 1));
            },
            *net, o);
        auto p = ml::predict_surface(in, *net, o);
        CHECK(f && p);
        if (f && p) {
            float worst = 0;
            for (std::size_t i = 0; i < vol.size(); ++i) worst = std::max(worst, std::fabs(f->data()[i] - p->data()[i]));
            CHECK(worst <= 1e-5f);
        }
        auto bad = ml::predict_surface_filled(d, [](s64, s64, s64, int P, float* out) { std::fill(out, out + P * P * P, 0.5f); }, *net, o);
        CHECK(!bad && bad.error().code == Errc::unsupported);
    }
    {  // output crop + tile filter through the header: the crop's dims, filtered tiles add nothing
        ml::InferOptions c = o;
        c.core_org = {32, 16, 8};
        c.core_ext = {64, 48, -1};
        auto p = ml::predict_surface(in, *net, c);
        CHECK(p && p->dims() == (Extent3{64, 48, 112}));
        ml::InferOptions t = o;
        t.tile_filter = [](s64 z0, s64, s64, s64) { return z0 >= 64; };
        auto q = ml::predict_surface(in, *net, t);
        CHECK(q.has_value());
        if (q) {  // planes below 32 are covered only by tiles starting at z 0: all zero
            bool zero = true;
            for (s64 i = 0; i < 32 * d.y * d.x; ++i) zero &= q->data()[i] == 0.0f;
            CHECK(zero);
        }
    }
    {  // the multi-GPU driver with two replicas (here on one device): z-slab shards, band sums
        auto n2 = ml::B200Net::load(weights, 64, 2);
        CHECK(n2.has_value());
        if (n2) {
            std::vector<ml::B200Net*> nets{&*net, &*n2};
            auto m = ml::predict_surface_multi(in, nets, o);
            auto p = ml::predict_surface(in, *net, o);
            CHECK(m && p);
            if (m && p) {
                float worst = 0;
                for (std::size_t i = 0; i < vol.size(); ++i) worst = std::max(worst, std::fabs(m->data()[i] - p->data()[i]));
                std::fprintf(stderr, "predict_surface_multi (2 replicas) vs predict_surface: max |d| %.3g\n", worst);
                CHECK(worst <= 1e-5f);
            }
            std::vector<ml::B200Net*> none;
            auto e = ml::predict_surface_multi(in, none, o);
            CHECK(!e && e.error().code == Errc::invalid_argument);
        }
    }
    std::printf("%s\n", fails ? "FAIL" : "ok");
    return fails ? 1 : 0;
}

static int gpu(const char* weights, const char* outpath) {
    const Extent3 d{100, 90, 140};  // smaller than two tiles on each axis, larger than one
    std::vector<u8> vol(static_cast<std::size_t>(d.count()));
    fx_spiral_params sp{12.0, 3.0, 170.0, 15.0, 40.0, 10.0, 1.0, 0.0};
    if (fx_synth_spiral(vol.data(), d.z, d.y, d.x, &sp, 5, 0, d.z) != 0) return 2;
    VolumeView<const u8> in(vol.data(), d);
    auto w1 = ml::predict_surface_window(in, weights);
    auto w2 = ml::predict_surface_window(in, weights);  // served by the cached net
    if (!w1 || !w2) {
        std::fprintf(stderr, "%s\n", (!w1 ? w1 : w2).error().message.c_str());
        return 3;
    }
    CHECK(w1->dims() == d && std::memcmp(w1->data(), w2->data(), vol.size()) == 0);
    auto net = ml::B200Net::load(weights, 128, 2);
    if (!net) return 4;
    ml::InferOptions o;
    o.patch = 128;
    o.overlap = 0.25;
    o.batch = 2;
    auto u = ml::predict_surface_u8(in, *net, o);
    auto p = ml::predict_surface(in, *net, o);
    if (!u || !p) return 5;
    // the u8 encoding of the f32 result, as the reference writes it
    std::size_t bad = 0;
    for (std::size_t i = 0; i < vol.size(); ++i) {
        const float c = std::min(std::max(p->data()[i], 0.f), 1.f);
        if (static_cast<u8>(c * 255.f + 0.5f) != u->data()[i]) ++bad;
    }
    CHECK(bad == 0);
    std::ofstream f(outpath, std::ios::binary);
    f.write(reinterpret_cast<const char*>(w1->data()), static_cast<std::streamsize>(vol.size()));
    f.write(reinterpret_cast<const char*>(u->data()), static_cast<std::streamsize>(vol.size()));
    f.write(reinterpret_cast<const char*>(vol.data()), static_cast<std::streamsize>(vol.size()));
    {  // GlobalAccum sink: the reference's constant round trip (18 chunks of exactly 153)
        auto g = ml::GlobalAccum::create({64, 0, 64}, {192, 128, 192}, 64, 0.5, 192);
        if (!g) return 6;
        std::vector<float> sp(64 * 64 * 64, 0.6f);
        const auto zs = fenix::ml::tile_starts(192, 64, 0.5), ys = fenix::ml::tile_starts(128, 64, 0.5);
        for (s64 z0 : zs)
            for (s64 y0 : ys)
                for (s64 x0 : zs) CHECK(g->scatter(64 + z0, y0, 64 + x0, 64, sp.data()).has_value());
        int chunks = 0, bad = 0;
        auto r = g->finalize_rows_below(g->chunk_rows(), [&](ChunkCoord c, const u8* blk) {
            ++chunks;
            if (c.z < 1 || c.x < 1) ++bad;
            for (int i = 0; i < 64 * 64 * 64; ++i) bad += blk[i] != 153;
        });
        CHECK(r.has_value() && chunks == 18 && bad == 0);
    }
    std::printf("%s\n", fails ? "FAIL" : "ok");
    return fails ? 1 : 0;
}

static int fxvol(const char* in, const char* out) {
    auto a = codec::VolumeArchive::open(in);
    CHECK(a.has_value());
    if (!a) return 1;
    const Extent3 d = a->dims();
    const auto prm = a->params();
    CHECK(a->src_dtype() == codec::DType::u8 && a->nlods() >= 1 && prm.q > 0.0f);
    auto b = codec::VolumeArchive::create(out, d, prm);
    CHECK(b.has_value());
    if (!b) return 1;
    Extent3 ld = d;
    int real = 0, zero = 0;
    for (uint32_t lod = 0; lod < a->nlods(); ++lod) {
        for (s64 z = 0; z < (ld.z + 63) / 64; ++z)
            for (s64 y = 0; y < (ld.y + 63) / 64; ++y)
                for (s64 x = 0; x < (ld.x + 63) / 64; ++x) {
                    const ChunkCoord c{z, y, x};
                    const auto cov = a->coverage(lod, c);
                    if (cov == codec::Coverage::Absent) continue;
                    auto p = a->chunk_payload(lod, c);
                    CHECK(p.has_value());
                    if (!p) continue;
                    CHECK((cov == codec::Coverage::Real) == !p->empty());
                    (cov == codec::Coverage::Real ? real : zero)++;
                    CHECK(b->write_chunk_payload(lod, c, *p).has_value());
                }
        ld = {(ld.z + 1) / 2, (ld.y + 1) / 2, (ld.x + 1) / 2};
    }
    CHECK(b->set_nlods(a->nlods()).has_value());
    CHECK(b->close().has_value());
    CHECK(a->close().has_value());
    CHECK(real > 0);
    // a missing file is not_found, a corrupt one decode_error
    auto m = codec::VolumeArchive::open(std::string(out) + ".missing");
    CHECK(!m && m.error().code == Errc::not_found);
    std::printf("%s %d %d\n", fails ? "FAIL" : "ok", real, zero);
    return fails ? 1 : 0;
}

// The checkpoint identity hash on the same inputs as oracle/ref_hash.cpp (the reference's own).
static int hash() {
    const int lens[] = {0, 1, 2, 3, 4, 7, 8, 15, 16, 17, 31, 32, 33, 100, 4096};
    for (int n : lens) {
        std::vector<u8> b(static_cast<std::size_t>(n));
        for (int i = 0; i < n; ++i) b[static_cast<std::size_t>(i)] = static_cast<u8>((i * 131 + 7) & 255);
        std::printf("bytes %d %llu %llu\n", n, static_cast<unsigned long long>(ml::hash64(b)),
                    static_cast<unsigned long long>(ml::hash64(b, 0x1234567890abcdefULL)));
    }
    std::vector<u8> chunk(1 << 20);
    u64 h = 0;
    for (int c = 0; c < 3; ++c) {
        const std::size_t n = c < 2 ? chunk.size() : 12345;
        for (std::size_t i = 0; i < n; ++i) chunk[i] = static_cast<u8>((i * 7 + static_cast<std::size_t>(c) * 13) & 255);
        h = ml::hash64({chunk.data(), n}, h);
    }
    std::printf("chain %llu\n", static_cast<unsigned long long>(h));
    return 0;
}

int main(int argc, char** argv) {
    if (argc >= 2 && std::string_view(argv[1]) == "hash") return hash();
    if (argc >= 2 && std::string_view(argv[1]) == "cpu") return cpu();
    if (argc >= 4 && std::string_view(argv[1]) == "fxvol") return fxvol(argv[2], argv[3]);
    if (argc >= 4 && std::string_view(argv[1]) == "gpu") return gpu(argv[2], argv[3]);
    if (argc >= 4 && std::string_view(argv[1]) == "stages") return stages(argv[2], argv[3]);
    std::fprintf(stderr, "usage: host_api_test cpu | gpu <weights> <out> | fxvol <in> <out>\n");
    return 2;
}
