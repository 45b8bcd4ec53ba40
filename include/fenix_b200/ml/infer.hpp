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
//   - the predict-surface stage argument grammar (src/ml/inference.cpp:369-420).
// Every computation runs on the GPU through the extern "C" ABI of fenix_b200.h. Options the device
// path does not implement (TTA, non-zscore normalisation, core crops, multi-scale, checkpoints,
// tile filters) return Errc::unsupported; there is no CPU fallback.
#pragma once

#include "fenix_b200.h"

#include <charconv>
#include <cstdint>
#include <cstring>
#include <expected>
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
    int tta = 0;  // <= 1: off (octahedral TTA is not implemented on this path)
    Index3 core_org{0, 0, 0};
    Extent3 core_ext{-1, -1, -1};  // whole input
    int batch = 3;                 // tiles per forward
};

// The options as the ABI struct, or unsupported/invalid_argument for what this path lacks.
[[nodiscard]] inline Expected<fx_infer_opts> to_fx(const InferOptions& o) {
    if (o.tta > 1) return err(Errc::unsupported, "InferOptions: test-time augmentation is not implemented on the B200 path");
    if (o.norm != Norm::zscore) return err(Errc::unsupported, "InferOptions: only zscore normalisation is implemented");
    if (o.core_ext.z >= 0 || o.core_ext.y >= 0 || o.core_ext.x >= 0)
        return err(Errc::unsupported, "InferOptions: core crops are not implemented on the B200 path");
    if (o.patch < 1 || o.batch < 1 || !(o.overlap >= 0.0 && o.overlap < 1.0))
        return err(Errc::invalid_argument, "InferOptions: bad patch, batch or overlap");
    if (o.channel < 0 || o.channel > 1) return err(Errc::invalid_argument, "InferOptions: channel must be 0 or 1");
    return fx_infer_opts{o.patch, o.overlap, o.channel, o.sigmoid ? 1 : 0, o.batch};
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
    Volume<f32> out(in.dims());
    if (auto r = detail::run(in, net, opt, out.data(), nullptr); !r) return std::unexpected(r.error());
    return out;
}

// The same, encoded (u8)(clamp(p, 0, 1) * 255 + 0.5).
[[nodiscard]] inline Expected<Volume<u8>> predict_surface_u8(VolumeView<const u8> in, B200Net& net,
                                                             const InferOptions& opt = {}) {
    Volume<u8> out(in.dims());
    if (auto r = detail::run(in, net, opt, nullptr, out.data()); !r) return std::unexpected(r.error());
    return out;
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

// Arguments of the predict-surface stage: <in> <weights> <out> [patch] [overlap] [tta] [batch],
// positional slots holding a key=value token are skipped, then key=value options. Keys this path
// adds: precision=f16|bf16|fp8 and device=N.
struct PredictArgs {
    std::string in, weights, out;
    InferOptions opt;
    bool batch_explicit = false;
    Precision precision = Precision::f16;
    int device = 0;
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
        } else if (k == "precision") {
            if (v == "f16" || v == "half") a.precision = Precision::f16;
            else if (v == "bf16") a.precision = Precision::bf16;
            else if (v == "fp8") a.precision = Precision::fp8;
            else return err(Errc::invalid_argument, "predict: precision must be f16, bf16 or fp8");
        } else if (k == "scales" || k == "rots" || k == "noise" || k == "offsets" || k == "ckpt") {
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
