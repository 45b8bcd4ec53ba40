// fenix_b200/ml/infer.hpp — header-only C++ host side of the B200 surface-prediction path.
//
// Mirrors the reference's torch-free ML surface so a caller switches by include and namespace:
//   - the error model Errc / Error / Expected<T> (src/core/error.hpp:19-43),
//   - Extent3 / Index3 / VolumeView<T> / Volume<T> (src/core/types.hpp:64-74, src/core/volume.hpp:19-120),
//   - ml::InferOptions, the subset the device path implements (src/ml/infer.hpp:38-103),
//   - the net operator concept batch()/patch()/classes() + forward on device tiles
//     (src/ml/trt_engine.hpp:35-106, src/ml/aoti_net.hpp:27-84),
//   - ml::predict_surface over a dense u8 volume (src/ml/infer.hpp:456-878 driven by the dense u8
//     filler of src/ml/inference.cpp:309-321) and its u8 encode (src/ml/inference.cpp:343-351),
//   - ml::predict_surface_window (src/ml/ml_api.hpp:16-24, src/ml/inference.cpp:914-962),
//   - the predict-surface stage argument grammar (src/ml/inference.cpp:369-420),
//   - ml::GlobalAccum, the global-grid accumulator with its z-sweep finalize and resume floor
//     (src/ml/global_accum.hpp:37-198), kept on the device.
//   - ml::predict_surface_filled with a caller's filler (src/ml/infer.hpp:452-458),
//   - InferOptions' normalisations (zscore / pct_minmax / unit255), output core crop and tile filter
//     (src/ml/infer.hpp:38-134, 462-472, 532-543),
// Every computation runs on the GPU through the extern "C" ABI of fenix_b200.h. Options the device
// path does not implement (multi-scale, rotation / noise / offset TTA, checkpoints) return
// Errc::unsupported; there is no CPU fallback.
#pragma once

#include "fenix_b200.h"
#include "fenix_b200/ml/tiling.hpp"

#include <algorithm>
#include <charconv>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <expected>
#include <functional>
#include <memory>
#include <mutex>
#include <span>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

namespace fenix_b200 {

using u8 = std::uint8_t;
using s64 = std::int64_t;
using u64 = std::uint64_t;
using f32 = float;

// Same enumerators in the same order as the reference's Errc; fx_status values equal them.
enum class Errc { ok = 0, invalid_argument, not_found, io_error, fetch_failed, decode_error, unsupported, unimplemented, internal };

struct Error {
    Errc code = Errc::internal;
    std::string message;
};

template <class T>
using Expected = std::expected<T, Error>;

[[nodiscard]] inline std::unexpected<Error> err(Errc code, std::string message) {
    return std::unexpected(Error{code, std::move(message)});
}
// A failed fx_* call as an Error: the status maps 1:1, the message is the thread's fx_last_error().
[[nodiscard]] inline std::unexpected<Error> err_status(fx_status st, std::string_view what) {
    std::string m(what);
    const char* e = fx_last_error();
    if (e && *e) m += std::string(": ") + e;
    return err(static_cast<Errc>(st), std::move(m));
}

struct Extent3 {
    s64 z = 0, y = 0, x = 0;
    [[nodiscard]] constexpr s64 count() const { return z * y * x; }
    friend constexpr bool operator==(Extent3, Extent3) = default;
};
struct Index3 {
    s64 z = 0, y = 0, x = 0;
    friend constexpr bool operator==(Index3, Index3) = default;
};
// Chunk coordinate = voxel >> 6 (64^3 chunks).
struct ChunkCoord {
    s64 z = 0, y = 0, x = 0;
    friend constexpr bool operator==(ChunkCoord, ChunkCoord) = default;
};

// Non-owning strided ZYX view (x fastest when contiguous).
template <class T>
class VolumeView {
public:
    constexpr VolumeView() = default;
    constexpr VolumeView(T* data, Extent3 dims, Index3 strides) : data_(data), dims_(dims), strides_(strides) {}
    constexpr VolumeView(T* data, Extent3 dims) : VolumeView(data, dims, contiguous_strides(dims)) {}
    static constexpr Index3 contiguous_strides(Extent3 d) { return {d.y * d.x, d.x, 1}; }
    [[nodiscard]] constexpr T* data() const { return data_; }
    [[nodiscard]] constexpr Extent3 dims() const { return dims_; }
    [[nodiscard]] constexpr Index3 strides() const { return strides_; }
    [[nodiscard]] constexpr bool contiguous() const { return strides_ == contiguous_strides(dims_); }
    constexpr T& operator()(s64 z, s64 y, s64 x) const { return data_[z * strides_.z + y * strides_.y + x * strides_.x]; }

private:
    T* data_ = nullptr;
    Extent3 dims_{};
    Index3 strides_{};
};

// Owning contiguous ZYX volume.
template <class T>
class Volume {
public:
    Volume() = default;
    explicit Volume(Extent3 dims)
        : dims_(dims), storage_(std::make_unique_for_overwrite<T[]>(static_cast<std::size_t>(dims.count()))) {}
    static Volume zeros(Extent3 dims) {
        Volume v(dims);
        std::memset(v.data(), 0, sizeof(T) * static_cast<std::size_t>(dims.count()));
        return v;
    }
    [[nodiscard]] T* data() { return storage_.get(); }
    [[nodiscard]] const T* data() const { return storage_.get(); }
    [[nodiscard]] Extent3 dims() const { return dims_; }
    [[nodiscard]] VolumeView<T> view() { return {data(), dims_}; }
    [[nodiscard]] VolumeView<const T> view() const { return {data(), dims_}; }

private:
    Extent3 dims_{};
    std::unique_ptr<T[]> storage_;
};

namespace ml {

enum class Norm { zscore, pct_minmax, unit255 };

// Tensor-core operand precision of the convolutions. f16 is the reference's own GPU precision
// (InferOptions::half); fp8 runs e4m3 with calibrated scales.
enum class Precision { bf16 = FX_PREC_BF16, fp8 = FX_PREC_FP8, f16 = FX_PREC_F16 };

struct InferOptions {
    int patch = 256;       // divisible by 2^(stages-1)
    double overlap = 0.5;  // step = (s64)(patch * (1 - overlap))
    bool half = true;      // 16-bit forward (f16 operands); false is not offered on this path
    int channel = 1;       // softmax channel to emit; ignored with sigmoid
    bool sigmoid = false;  // 1-class head -> sigmoid
    Norm norm = Norm::zscore;
    int tta = 0;  // <= 1: off; else the first min(tta, 48) octahedral symmetries, averaged
    // Output crop: the returned volume covers only [core_org, core_org + core_ext) of the input;
    // tiles still read the whole input, a tile that does not reach the core is not run. A negative
    // extent component = to the end of the input (the default: no crop).
    Index3 core_org{0, 0, 0};
    Extent3 core_ext{-1, -1, -1};
    int batch = 3;                 // tiles per forward
    // A tile (origin z0, y0, x0, side patch) runs only if this returns true (src/ml/infer.hpp:102);
    // called on the calling thread while the tile list is built. Empty = every tile.
    std::function<bool(s64 z0, s64 y0, s64 x0, s64 patch)> tile_filter{};
    // Tiles whose input voxels all hold one value are not run (they add nothing to the blend) —
    // predict-scroll's constant-input filter (src/ml/inference.cpp:1487-1496, 1885-1900), evaluated
    // on the device.
    bool skip_constant = false;
    // Resumable prediction (src/ml/infer.hpp:78-96): checkpoint file (empty = off), the cadence in
    // tiles, and the identity of the weights / input it belongs to (see weights_hash64 below).
    std::string ckpt_path{};
    long ckpt_every = 128;
    u64 weights_hash = 0;
    u64 input_hash = 0;
};

// The reference's 64-bit identity hash (src/core/hash.hpp:36-59): wyhash-style mixing (Wang Yi's
// public-domain wyhash: a 64 x 64 -> 128-bit multiply folded by xor, 16-byte rounds, the 4-16 and
// 1-3 byte tails), restated so that a checkpoint's weights / input identity equals the reference's
// and either side resumes the other's file.
inline u64 hash64(std::span<const u8> data, u64 seed = 0) {
    constexpr u64 p0 = 0xa0761d6478bd642fULL, p1 = 0xe7037ed1a0b428dbULL;
    auto mix = [](u64 a, u64 b) {
        const __uint128_t r = static_cast<__uint128_t>(a) * b;
        return static_cast<u64>(r) ^ static_cast<u64>(r >> 64);
    };
    auto r64 = [](const u8* q) {
        u64 v;
        std::memcpy(&v, q, 8);
        return v;
    };
    auto r32 = [](const u8* q) {
        uint32_t v;
        std::memcpy(&v, q, 4);
        return static_cast<u64>(v);
    };
    const u8* q = data.data();
    std::size_t len = data.size();
    u64 a = 0, b = 0;
    seed ^= mix(seed ^ p0, p1);
    if (len <= 16) {
        if (len >= 4) {
            a = (r32(q) << 32) | r32(q + ((len >> 3) << 2));
            b = (r32(q + len - 4) << 32) | r32(q + len - 4 - ((len >> 3) << 2));
        } else if (len > 0) {
            a = (static_cast<u64>(q[0]) << 16) | (static_cast<u64>(q[len >> 1]) << 8) | q[len - 1];
        }
    } else {
        std::size_t i = len;
        while (i > 16) {
            seed = mix(r64(q) ^ p1, r64(q + 8) ^ seed);
            q += 16;
            i -= 16;
        }
        a = r64(q + i - 16);
        b = r64(q + i - 8);
    }
    return mix(p1 ^ len, mix(a ^ p1, b ^ seed));
}

// A weights file's checkpoint identity: hash64 chained over its bytes in 1 MiB chunks, as the
// reference's predict computes it (src/ml/inference.cpp:256-274); 0 when it cannot be read.
inline u64 weights_hash64(const std::string& path) {
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return 0;
    std::vector<u8> chunk(1 << 20);
    u64 h = 0;
    for (;;) {
        const std::size_t n = std::fread(chunk.data(), 1, chunk.size(), f);
        if (n == 0) break;
        h = hash64({chunk.data(), n}, h);
    }
    std::fclose(f);
    return h;
}

namespace detail {
inline int tile_filter_trampoline(int64_t z0, int64_t y0, int64_t x0, int64_t p, void* user) {
    const auto* f = static_cast<const std::function<bool(s64, s64, s64, s64)>*>(user);
    try {
        return (*f)(z0, y0, x0, p) ? 1 : 0;
    } catch (...) {
        return 1;  // a filter that fails keeps its tile
    }
}
}  // namespace detail

// The options as the ABI struct, or invalid_argument for what cannot hold. The struct refers to
// o.tile_filter: keep `o` alive while it is in use.
[[nodiscard]] inline Expected<fx_infer_opts> to_fx(const InferOptions& o) {
    if (o.patch < 1 || o.batch < 1 || !(o.overlap >= 0.0 && o.overlap < 1.0))
        return err(Errc::invalid_argument, "InferOptions: bad patch, batch or overlap");
    if (o.channel < 0 || o.channel > 1) return err(Errc::invalid_argument, "InferOptions: channel must be 0 or 1");
    fx_infer_opts f{};
    f.patch = o.patch;
    f.overlap = o.overlap;
    f.channel = o.channel;
    f.sigmoid = o.sigmoid ? 1 : 0;
    f.batch = o.batch;
    f.tta = o.tta;
    f.norm = o.norm == Norm::pct_minmax ? FX_NORM_PCT_MINMAX : (o.norm == Norm::unit255 ? FX_NORM_UNIT255 : FX_NORM_ZSCORE);
    f.skip_constant = o.skip_constant ? 1 : 0;
    f.core_org[0] = o.core_org.z;
    f.core_org[1] = o.core_org.y;
    f.core_org[2] = o.core_org.x;
    if (o.core_ext.z == 0 || o.core_ext.y == 0 || o.core_ext.x == 0)
        return err(Errc::invalid_argument, "InferOptions: an empty output crop");
    // "to the end" is a negative component here and a non-positive one in the ABI
    f.core_ext[0] = std::max<s64>(o.core_ext.z, 0);
    f.core_ext[1] = std::max<s64>(o.core_ext.y, 0);
    f.core_ext[2] = std::max<s64>(o.core_ext.x, 0);
    if (o.tile_filter) {
        f.tile_filter = &detail::tile_filter_trampoline;
        f.tile_filter_user = const_cast<std::function<bool(s64, s64, s64, s64)>*>(&o.tile_filter);
    }
    if (!o.ckpt_path.empty()) {
        f.ckpt_path = o.ckpt_path.c_str();
        f.ckpt_every = o.ckpt_every;
        f.weights_hash = o.weights_hash;
        f.input_hash = o.input_hash;
    }
    return f;
}

// The output dims of a prediction over an input of dims d with opt's crop (src/ml/infer.hpp:462-472).
[[nodiscard]] inline Extent3 output_dims(Extent3 d, const InferOptions& o) {
    auto ax = [](s64 org, s64 ext, s64 n) {
        const s64 c = std::clamp<s64>(org, 0, n);
        return ext < 0 ? n - c : std::min(ext, n - c);
    };
    return {ax(o.core_org.z, o.core_ext.z, d.z), ax(o.core_org.y, o.core_ext.y, d.y), ax(o.core_org.x, o.core_ext.x, d.x)};
}

// One net on one device (the operator concept of the reference's TrtNet / AotiNet).
class B200Net {
public:
    B200Net() = default;
    B200Net(const B200Net&) = delete;
    B200Net& operator=(const B200Net&) = delete;
    B200Net(B200Net&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
    B200Net& operator=(B200Net&& o) noexcept {
        if (this != &o) {
            reset();
            h_ = std::exchange(o.h_, nullptr);
        }
        return *this;
    }
    ~B200Net() { reset(); }

    [[nodiscard]] static Expected<B200Net> load(const std::string& fxweights, int patch, int max_batch,
                                                Precision precision = Precision::f16, int device = 0) {
        B200Net n;
        const fx_status st =
            fx_net_create(fxweights.c_str(), patch, max_batch, static_cast<fx_precision>(precision), device, &n.h_);
        if (st != FX_OK) return err_status(st, "B200Net::load(" + fxweights + ")");
        return n;
    }
    [[nodiscard]] int batch() const { return fx_net_max_batch(h_); }
    [[nodiscard]] int patch() const { return fx_net_patch(h_); }
    [[nodiscard]] int classes() const { return fx_net_classes(h_); }
    [[nodiscard]] fx_net* handle() const { return h_; }
    explicit operator bool() const { return h_ != nullptr; }

    // fp8 nets: per-tensor activation scales from n host patches [n][P][P][P].
    [[nodiscard]] Expected<void> calibrate(std::span<const u8> patches, int n) {
        const s64 P = patch();
        if (n < 1 || static_cast<s64>(patches.size()) < n * P * P * P)
            return err(Errc::invalid_argument, "B200Net::calibrate: need n patches of P^3 voxels");
        const fx_status st = fx_net_calibrate(h_, patches.data(), n);
        if (st != FX_OK) return err_status(st, "B200Net::calibrate");
        return {};
    }
    // nb device u8 tiles [nb][P][P][P] -> class probability [nb][P][P][P] f32 on the device.
    [[nodiscard]] Expected<void> forward(const u8* dev_tiles, int nb, float* dev_prob, int channel = 1,
                                         bool sigmoid = false, void* stream = nullptr) {
        const fx_status st = fx_net_forward(h_, dev_tiles, nb, dev_prob, channel, sigmoid ? 1 : 0, stream);
        if (st != FX_OK) return err_status(st, "B200Net::forward");
        return {};
    }

private:
    void reset() {
        if (h_) fx_net_destroy(h_);
        h_ = nullptr;
    }
    fx_net* h_ = nullptr;
};

namespace detail {
// The input as one contiguous host buffer: the view itself when contiguous, else a gathered copy.
inline const u8* contiguous_input(VolumeView<const u8> in, std::vector<u8>& tmp) {
    if (in.contiguous()) return in.data();
    const Extent3 d = in.dims();
    tmp.resize(static_cast<std::size_t>(d.count()));
    std::size_t i = 0;
    for (s64 z = 0; z < d.z; ++z)
        for (s64 y = 0; y < d.y; ++y)
            for (s64 x = 0; x < d.x; ++x) tmp[i++] = in(z, y, x);
    return tmp.data();
}

inline Expected<void> run(VolumeView<const u8> in, B200Net& net, const InferOptions& opt, float* prob, u8* u8out) {
    if (!net) return err(Errc::invalid_argument, "predict_surface: empty net");
    const Extent3 d = in.dims();
    if (d.z < 1 || d.y < 1 || d.x < 1 || !in.data()) return err(Errc::invalid_argument, "predict_surface: empty volume");
    if (opt.patch != net.patch())
        return err(Errc::invalid_argument, "predict_surface: patch " + std::to_string(opt.patch) +
                                               " differs from the net's " + std::to_string(net.patch()));
    auto o = to_fx(opt);
    if (!o) return std::unexpected(o.error());
    if (o->batch > net.batch()) o->batch = net.batch();
    std::vector<u8> tmp;
    const u8* src = contiguous_input(in, tmp);
    const fx_status st = fx_predict_volume(net.handle(), src, d.z, d.y, d.x, &*o, prob, u8out);
    if (st != FX_OK) return err_status(st, "predict_surface");
    return {};
}
}  // namespace detail

// Sliding-window surface probability over a u8 volume: per-tile zscore, Gaussian blend,
// normalise by the factorised weight (same dims as the input).
[[nodiscard]] inline Expected<Volume<f32>> predict_surface(VolumeView<const u8> in, B200Net& net,
                                                           const InferOptions& opt = {}) {
    Volume<f32> out(output_dims(in.dims(), opt));
    if (auto r = detail::run(in, net, opt, out.data(), nullptr); !r) return std::unexpected(r.error());
    return out;
}

// The same, encoded (u8)(clamp(p, 0, 1) * 255 + 0.5).
[[nodiscard]] inline Expected<Volume<u8>> predict_surface_u8(VolumeView<const u8> in, B200Net& net,
                                                             const InferOptions& opt = {}) {
    Volume<u8> out(output_dims(in.dims(), opt));
    if (auto r = detail::run(in, net, opt, nullptr, out.data()); !r) return std::unexpected(r.error());
    return out;
}

// The same over several GPUs (the reference's one model replica per visible device,
// src/ml/inference.cpp:1129-1188): the volume is split into z-slabs by contiguous ranges of the
// tile grid, one host thread per net predicts its slab on its device, each owner adds the tile
// overlap bands its neighbours accumulated by reading their device memory directly (peer access
// over NVLink / NVSwitch, no NCCL), finalises the planes it owns and copies them to the output.
// Equals predict_surface up to the order of the band sums. The nets share weights, precision and
// (fp8) activation scales and schedule; two nets may share a device. No output crop.
namespace detail {
inline Expected<void> run_multi(VolumeView<const u8> in, std::span<B200Net* const> nets, const InferOptions& opt,
                                float* prob, u8* u8out) {
    if (nets.empty()) return err(Errc::invalid_argument, "predict_surface_multi: no nets");
    std::vector<fx_net*> h;
    int batch = 1 << 30;
    for (B200Net* n : nets) {
        if (!n || !*n) return err(Errc::invalid_argument, "predict_surface_multi: empty net");
        if (opt.patch != n->patch()) return err(Errc::invalid_argument, "predict_surface_multi: patch differs from a net's");
        h.push_back(n->handle());
        batch = std::min(batch, n->batch());
    }
    const Extent3 d = in.dims();
    if (d.z < 1 || d.y < 1 || d.x < 1 || !in.data()) return err(Errc::invalid_argument, "predict_surface_multi: empty volume");
    auto o = to_fx(opt);
    if (!o) return std::unexpected(o.error());
    if (o->batch > batch) o->batch = batch;
    std::vector<u8> tmp;
    const u8* src = contiguous_input(in, tmp);
    const fx_status st =
        fx_predict_volume_multi(h.data(), static_cast<int>(h.size()), src, d.z, d.y, d.x, &*o, prob, u8out);
    if (st != FX_OK) return err_status(st, "predict_surface_multi");
    return {};
}
}  // namespace detail

[[nodiscard]] inline Expected<Volume<f32>> predict_surface_multi(VolumeView<const u8> in, std::span<B200Net* const> nets,
                                                                 const InferOptions& opt = {}) {
    Volume<f32> out(in.dims());
    if (auto r = detail::run_multi(in, nets, opt, out.data(), nullptr); !r) return std::unexpected(r.error());
    return out;
}

[[nodiscard]] inline Expected<Volume<u8>> predict_surface_multi_u8(VolumeView<const u8> in,
                                                                   std::span<B200Net* const> nets,
                                                                   const InferOptions& opt = {}) {
    Volume<u8> out(in.dims());
    if (auto r = detail::run_multi(in, nets, opt, nullptr, out.data()); !r) return std::unexpected(r.error());
    return out;
}

// predict_surface_filled (src/ml/infer.hpp:452-458): the input comes from a caller's filler,
// fill(z0, y0, x0, P, float* out) writing the P^3 patch at that origin (out of the volume it must
// clamp, as the reference's fillers do). The device path normalises u8 levels exactly, so every
// filled value must be an integer in [0, 255] (the reference's u8 sources); anything else is
// Errc::unsupported. The patches are gathered into a dense u8 volume of dims d on the host, which
// is then predicted on the device like predict_surface.
template <class Filler>
[[nodiscard]] inline Expected<Volume<f32>> predict_surface_filled(Extent3 d, Filler&& fill, B200Net& net,
                                                                  const InferOptions& opt = {}) {
    if (opt.patch % 64 != 0) return err(Errc::invalid_argument, "patch must be divisible by 64");
    if (d.z < 1 || d.y < 1 || d.x < 1) return err(Errc::invalid_argument, "predict_surface_filled: empty volume");
    const int P = opt.patch;
    Volume<u8> vol(d);
    std::vector<float> patch(static_cast<std::size_t>(P) * P * P);
    const std::vector<s64> zs = fenix::ml::tile_starts(d.z, P, opt.overlap), ys = fenix::ml::tile_starts(d.y, P, opt.overlap),
                           xs = fenix::ml::tile_starts(d.x, P, opt.overlap);
    for (s64 z0 : zs)
        for (s64 y0 : ys)
            for (s64 x0 : xs) {
                fill(z0, y0, x0, P, patch.data());
                for (s64 z = 0; z < P && z0 + z < d.z; ++z)
                    for (s64 y = 0; y < P && y0 + y < d.y; ++y)
                        for (s64 x = 0; x < P && x0 + x < d.x; ++x) {
                            const float v = patch[static_cast<std::size_t>((z * P + y) * P + x)];
                            if (!(v >= 0.0f && v <= 255.0f) || v != static_cast<float>(static_cast<int>(v)))
                                return err(Errc::unsupported, "predict_surface_filled: filled values must be u8 levels");
                            vol.view()(z0 + z, y0 + y, x0 + x) = static_cast<u8>(v);
                        }
            }
    return predict_surface(static_cast<const Volume<u8>&>(vol).view(), net, opt);
}

// One resident u8 window -> u8 sheet probability, same dims: patch 128, overlap 0.25, f16,
// zscore, softmax channel 1. The net is loaded once per weights path (on device 0) and reused;
// calls are serialised by a process-wide mutex.
[[nodiscard]] inline Expected<Volume<u8>> predict_surface_window(VolumeView<const u8> ct,
                                                                 const std::string& weights_path) {
    struct Cache {
        std::string path;
        B200Net net;
    };
    static Cache cache;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    InferOptions opt;
    opt.patch = 128;
    opt.overlap = 0.25;
    if (!cache.net || cache.path != weights_path) {
        cache.net = B200Net{};
        auto n = B200Net::load(weights_path, opt.patch, opt.batch, Precision::f16, 0);
        if (!n) return std::unexpected(n.error());
        cache.net = std::move(*n);
        cache.path = weights_path;
    }
    return predict_surface_u8(ct, cache.net, opt);
}

// The global tile grid of predict-scroll over a 64-aligned bbox with its accumulator on the
// device (fx_gaccum_*): scatter tiles or run whole tile rows through a net, then finalize chunk
// rows below a z-front; finalize_rows_below hands every 64^3 chunk of those rows to
// sink(ChunkCoord /*archive coordinates*/, const u8* /*64^3 ZYX*/), voxels past the bbox as 0.
class GlobalAccum {
public:
    static constexpr s64 T = 64;
    GlobalAccum() = default;
    GlobalAccum(const GlobalAccum&) = delete;
    GlobalAccum& operator=(const GlobalAccum&) = delete;
    GlobalAccum(GlobalAccum&& o) noexcept
        : h_(std::exchange(o.h_, nullptr)), org_(o.org_), ext_(o.ext_), patch_(o.patch_), overlap_(o.overlap_) {}
    GlobalAccum& operator=(GlobalAccum&& o) noexcept {
        if (this != &o) {
            if (h_) fx_gaccum_destroy(h_);
            h_ = std::exchange(o.h_, nullptr);
            org_ = o.org_;
            ext_ = o.ext_;
            patch_ = o.patch_;
            overlap_ = o.overlap_;
        }
        return *this;
    }
    ~GlobalAccum() {
        if (h_) fx_gaccum_destroy(h_);
    }

    // window_planes: accumulator planes kept on the device (0 = patch + 64, enough for a sweep
    // that finalizes the chunk rows below each tile row before running it).
    [[nodiscard]] static Expected<GlobalAccum> create(Index3 org, Extent3 ext, int patch, double overlap,
                                                      s64 window_planes = 0, int device = 0) {
        GlobalAccum a;
        const int64_t o[3] = {org.z, org.y, org.x}, e[3] = {ext.z, ext.y, ext.x};
        const fx_status st = fx_gaccum_create(o, e, patch, overlap, window_planes, device, &a.h_);
        if (st != FX_OK) return err_status(st, "GlobalAccum::create");
        a.org_ = org;
        a.ext_ = ext;
        a.patch_ = patch;
        a.overlap_ = overlap;
        return a;
    }
    [[nodiscard]] s64 chunk_rows() const { return fx_gaccum_chunk_rows(h_); }
    [[nodiscard]] s64 floor_row() const { return fx_gaccum_floor_row(h_); }
    [[nodiscard]] s64 tile_rows() const { return fx_gaccum_tile_rows(h_); }
    [[nodiscard]] s64 row_start(s64 zi) const { return fx_gaccum_row_start(h_, zi); }
    [[nodiscard]] Expected<void> set_floor_row(s64 floor_row) {
        const fx_status st = fx_gaccum_set_floor_row(h_, floor_row);
        if (st != FX_OK) return err_status(st, "GlobalAccum::set_floor_row");
        return {};
    }
    // Gaussian-blend one P^3 probability tile at scroll coordinates (P = the grid's patch).
    [[nodiscard]] Expected<void> scatter(s64 z0, s64 y0, s64 x0, int P, const float* sp) {
        if (P != patch_) return err(Errc::invalid_argument, "GlobalAccum::scatter: patch differs from the grid's");
        const fx_status st = fx_gaccum_scatter(h_, z0, y0, x0, sp);
        if (st != FX_OK) return err_status(st, "GlobalAccum::scatter");
        return {};
    }
    // All tiles of tile row zi through `net`; planes = bbox-local input planes
    // [row_start(zi), min(row_start(zi) + patch, ext.z)), [n][ext.y][ext.x].
    [[nodiscard]] Expected<void> predict_row(B200Net& net, s64 zi, const u8* planes, const InferOptions& opt) {
        auto o = to_fx(opt);
        if (!o) return std::unexpected(o.error());
        const fx_status st = fx_gaccum_predict_row(h_, net.handle(), zi, planes, &*o);
        if (st != FX_OK) return err_status(st, "GlobalAccum::predict_row");
        return {};
    }
    template <class Sink>
    [[nodiscard]] Expected<void> finalize_rows_below(s64 row_lim, Sink&& sink) {
        const s64 r0 = floor_row(), r1 = std::min(row_lim, chunk_rows());
        if (r1 <= r0) return {};
        const s64 z0 = r0 * T, z1 = std::min(r1 * T, ext_.z), plane = ext_.y * ext_.x;
        std::vector<u8> planes(static_cast<std::size_t>((z1 - z0) * plane));
        int64_t n = 0;
        const fx_status st = fx_gaccum_finalize_below(h_, row_lim, planes.data(), static_cast<int64_t>(planes.size()), &n);
        if (st != FX_OK) return err_status(st, "GlobalAccum::finalize_rows_below");
        std::vector<u8> blk(static_cast<std::size_t>(T * T * T));
        const s64 ncy = (ext_.y + T - 1) / T, ncx = (ext_.x + T - 1) / T;
        for (s64 cz = r0; cz < r1; ++cz)
            for (s64 cy = 0; cy < ncy; ++cy)
                for (s64 cx = 0; cx < ncx; ++cx) {
                    std::fill(blk.begin(), blk.end(), u8{0});
                    for (s64 z = 0; z < T && cz * T + z < z1; ++z)
                        for (s64 y = 0; y < T && cy * T + y < ext_.y; ++y) {
                            const s64 xs = std::min<s64>(T, ext_.x - cx * T);
                            const u8* src = planes.data() + ((cz * T + z - z0) * ext_.y + cy * T + y) * ext_.x + cx * T;
                            std::memcpy(blk.data() + (z * T + y) * T, src, static_cast<std::size_t>(xs));
                        }
                    sink(ChunkCoord{org_.z / T + cz, org_.y / T + cy, org_.x / T + cx}, static_cast<const u8*>(blk.data()));
                }
        return {};
    }

private:
    fx_gaccum* h_ = nullptr;
    Index3 org_{};
    Extent3 ext_{};
    int patch_ = 0;
    double overlap_ = 0.5;
};

// Arguments of the predict-surface stage: <in> <weights> <out> [patch] [overlap] [tta] [batch],
// positional slots holding a key=value token are skipped, then key=value options. Keys this path
// adds: precision=f16|bf16|fp8, device=N and gpus=N (devices [device, device + N), one replica each).
struct PredictArgs {
    std::string in, weights, out;
    InferOptions opt;
    bool batch_explicit = false;
    Precision precision = Precision::f16;
    int device = 0;
    int gpus = 1;
};

[[nodiscard]] inline Expected<PredictArgs> parse_predict_args(std::span<const std::string_view> args,
                                                              std::string_view name = "predict-surface") {
    if (args.size() < 3)
        return err(Errc::invalid_argument, std::string("usage: ") + std::string(name) +
                                               " <in.fxvol> <weights.fxweights> <out.fxvol> [patch] [overlap] [tta] [batch]");
    PredictArgs a;
    a.in = std::string(args[0]);
    a.weights = std::string(args[1]);
    a.out = std::string(args[2]);
    auto is_kw = [](std::string_view s) { return s.find('=') != std::string_view::npos; };
    auto to_int = [](std::string_view s, int& out) -> Expected<void> {
        int v = 0;
        const auto r = std::from_chars(s.data(), s.data() + s.size(), v);
        if (r.ec != std::errc{} || r.ptr != s.data() + s.size())
            return err(Errc::invalid_argument, "predict: not an integer: " + std::string(s));
        out = v;
        return {};
    };
    auto to_double = [](std::string_view s, double& out) -> Expected<void> {
        double v = 0;
        const auto r = std::from_chars(s.data(), s.data() + s.size(), v);
        if (r.ec != std::errc{} || r.ptr != s.data() + s.size())
            return err(Errc::invalid_argument, "predict: not a number: " + std::string(s));
        out = v;
        return {};
    };
    if (args.size() >= 4 && !is_kw(args[3]))
        if (auto r = to_int(args[3], a.opt.patch); !r) return std::unexpected(r.error());
    if (args.size() >= 5 && !is_kw(args[4]))
        if (auto r = to_double(args[4], a.opt.overlap); !r) return std::unexpected(r.error());
    if (args.size() >= 6 && !is_kw(args[5]))
        if (auto r = to_int(args[5], a.opt.tta); !r) return std::unexpected(r.error());
    if (args.size() >= 7 && !is_kw(args[6])) {
        if (auto r = to_int(args[6], a.opt.batch); !r) return std::unexpected(r.error());
        a.batch_explicit = true;
    }
    for (std::size_t i = 3; i < args.size(); ++i) {
        const std::string_view t = args[i];
        if (!is_kw(t)) {
            if (i >= 7) return err(Errc::invalid_argument, "predict: unexpected argument: " + std::string(t));
            continue;
        }
        const std::string_view k = t.substr(0, t.find('=')), v = t.substr(t.find('=') + 1);
        if (k == "patch") {
            if (auto r = to_int(v, a.opt.patch); !r) return std::unexpected(r.error());
        } else if (k == "overlap") {
            if (auto r = to_double(v, a.opt.overlap); !r) return std::unexpected(r.error());
        } else if (k == "tta") {
            if (auto r = to_int(v, a.opt.tta); !r) return std::unexpected(r.error());
        } else if (k == "batch") {
            if (auto r = to_int(v, a.opt.batch); !r) return std::unexpected(r.error());
            a.batch_explicit = true;
        } else if (k == "device") {
            if (auto r = to_int(v, a.device); !r) return std::unexpected(r.error());
        } else if (k == "gpus") {
            if (auto r = to_int(v, a.gpus); !r) return std::unexpected(r.error());
            if (a.gpus < 1) return err(Errc::invalid_argument, "predict: gpus must be >= 1");
        } else if (k == "precision") {
            if (v == "f16" || v == "half") a.precision = Precision::f16;
            else if (v == "bf16") a.precision = Precision::bf16;
            else if (v == "fp8") a.precision = Precision::fp8;
            else return err(Errc::invalid_argument, "predict: precision must be f16, bf16 or fp8");
        } else if (k == "ckpt") {
            a.opt.ckpt_path = std::string(v);
        } else if (k == "ckpt_every") {
            int e = 0;
            if (auto r = to_int(v, e); !r) return std::unexpected(r.error());
            a.opt.ckpt_every = e;
        } else if (k == "scales" || k == "rots" || k == "noise" || k == "offsets") {
            return err(Errc::unsupported, "predict: " + std::string(k) + "= is not implemented on the B200 path");
        } else {
            return err(Errc::invalid_argument, "predict: unknown option: " + std::string(k));
        }
    }
    if (auto o = to_fx(a.opt); !o) return std::unexpected(o.error());
    return a;
}

}  // namespace ml
}  // namespace fenix_b200
