// Exercises the header-only host API (fenix_b200/ml/infer.hpp) against the C ABI.
//   host_api_test cpu                   — argument grammar, option checks, views, error mapping
//   host_api_test gpu <weights> <out>   — predict_surface_window and predict_surface_u8 on a
//                                         synthetic window; writes both outputs to <out>
//   host_api_test fxvol <in> <out>      — codec::VolumeArchive: open an archive, check its metadata
//                                         and rewrite every chunk payload of every LOD to <out>
#include "fenix_b200/codec/archive.hpp"
#include "fenix_b200/ml/infer.hpp"
#include "fenix_b200/ml/tiling.hpp"
#include "fenix_b200_synth.h"

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
    {
        ml::InferOptions o;
        o.norm = ml::Norm::pct_minmax;
        CHECK(ml::to_fx(o).error().code == Errc::unsupported);
        o = {};
        o.core_ext = {64, 64, 64};
        CHECK(ml::to_fx(o).error().code == Errc::unsupported);
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

int main(int argc, char** argv) {
    if (argc >= 2 && std::string_view(argv[1]) == "cpu") return cpu();
    if (argc >= 4 && std::string_view(argv[1]) == "fxvol") return fxvol(argv[2], argv[3]);
    if (argc >= 4 && std::string_view(argv[1]) == "gpu") return gpu(argv[2], argv[3]);
    std::fprintf(stderr, "usage: host_api_test cpu | gpu <weights> <out> | fxvol <in> <out>\n");
    return 2;
}
